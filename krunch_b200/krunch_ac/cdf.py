"""Probability -> integer CDF (krunch_ac/cdf.py:22-74), computed on the GPU.

Same rule: count = floor(p * (T - V)) + 1, the deficit goes to the argmax bin
(smallest index on ties), cdf = [0, cumsum].  The row sum runs in the
kernel's fixed order, so results are reproducible bit for bit on any batch
size (the numpy reference's pairwise sum may differ in a last bit).
"""
from __future__ import annotations

import numpy as np
import torch

from .. import _native as N

CDF_PRECISION = 24
T = 1 << CDF_PRECISION


def probs_to_cdf(probs, bits: int = CDF_PRECISION):
    """(N, V) probabilities -> (N, V+1) CDF.  numpy in -> numpy uint32 out
    (the reference's return type); CUDA tensor in -> int32 CUDA tensor out."""
    as_numpy = isinstance(probs, np.ndarray)
    p = torch.as_tensor(probs)
    if p.dim() == 1:
        p = p.reshape(1, -1)
    if not p.is_cuda:
        if not torch.cuda.is_available():
            raise RuntimeError("krunch_b200.krunch_ac needs a CUDA device")
        p = p.cuda()
    p = p.to(torch.float32).contiguous()
    n, V = p.shape
    if V >= (1 << bits):
        raise ValueError(f"vocab size {V} must be < T={1 << bits}")
    out = torch.empty((n, V + 1), dtype=torch.int32, device=p.device)
    N.call("kb_cdf_from_probs", p.data_ptr(), n, V, bits, out.data_ptr(), N.stream_ptr(p.device))
    if as_numpy:
        return out.cpu().numpy().view(np.uint32)
    return out
