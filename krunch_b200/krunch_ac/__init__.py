"""GPU CDF + range coder API with the names of the reference's krunch_ac package
(krunch_ac/__init__.py:21-32).

``probs_to_cdf`` and ``CDF_PRECISION`` keep their meaning; the coder entry
points ``encode`` / ``decode`` run the GPU kernels.  (The reference's
``encode_cpu`` / ``decode_cpu`` are its CPU specification; this package has no
CPU code path.)
"""
from .cdf import CDF_PRECISION, T, probs_to_cdf
from .gpu_encode import decode, encode, encode_chunk_gpu, probs_to_cdf_gpu

__all__ = ["probs_to_cdf", "CDF_PRECISION", "T", "encode", "decode", "probs_to_cdf_gpu",
           "encode_chunk_gpu"]
