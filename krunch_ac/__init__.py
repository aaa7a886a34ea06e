"""Import name of the reference's ``krunch_ac`` package (krunch_ac/__init__.py:21-32)
mapped onto krunch_b200.krunch_ac.

``probs_to_cdf`` and ``CDF_PRECISION`` keep their meaning.  ``encode_cpu`` /
``decode_cpu`` keep their signatures — ``(cdf [N, V+1], symbols [N]) -> bytes``
and ``(bytes, cdfs [N, V+1]) -> symbols`` — and their bytes (the GPU coder is
bit-exact with the reference's CPU coder), but run on the GPU: this build has
no CPU code path.
"""
from krunch_b200.krunch_ac import (CDF_PRECISION, T, decode, encode, encode_chunk_gpu,  # noqa: F401
                                   probs_to_cdf, probs_to_cdf_gpu)

encode_cpu = encode
decode_cpu = decode

__all__ = ["probs_to_cdf", "CDF_PRECISION", "encode_cpu", "decode_cpu"]
