"""GPU encode / decode drivers (krunch_ac/gpu_encode.py:22-102 surface)."""
from __future__ import annotations

import numpy as np
import torch

from .. import _native as N
from .cdf import CDF_PRECISION, probs_to_cdf


def probs_to_cdf_gpu(probs: torch.Tensor, bits: int = CDF_PRECISION) -> torch.Tensor:
    assert probs.is_cuda and probs.dim() == 2
    return probs_to_cdf(probs, bits)


def _bits_of(cdf: torch.Tensor) -> int:
    T = int(cdf[0, -1].item())
    if T <= 0 or T & (T - 1):
        raise ValueError(f"CDF total {T} is not a power of two")
    return T.bit_length() - 1


def encode(cdf, symbols) -> bytes:
    """One stream: CDF [N, V+1] (cdf[:,V] = 2^bits) + symbols [N] -> bytes."""
    c = torch.as_tensor(np.asarray(cdf).astype(np.int32) if isinstance(cdf, np.ndarray) else cdf)
    c = c.cuda().to(torch.int32).contiguous()
    s = torch.as_tensor(symbols).cuda().to(torch.int32).contiguous()
    n = c.shape[0]
    bits = _bits_of(c) if n else CDF_PRECISION
    cap = n * (bits + 2) // 8 + 64
    out = torch.zeros(cap, dtype=torch.uint8, device=c.device)
    st = torch.empty(4, dtype=torch.int32, device=c.device)
    sp = N.stream_ptr(c.device)
    N.call("kb_coder_encode_init", st.data_ptr(), 1, sp)
    if n:
        N.call("kb_coder_encode_cdf", c.data_ptr(), c.shape[1], s.data_ptr(), n, bits,
               out.data_ptr(), cap, st.data_ptr(), sp)
    N.call("kb_coder_encode_finalize", out.data_ptr(), cap, None, st.data_ptr(), 1, sp)
    nbits = int(st[3].item()) & 0xFFFFFFFF
    nbytes = (nbits + 7) // 8
    if nbytes > cap:
        raise RuntimeError("encoded stream exceeded its buffer")
    return out[:nbytes].cpu().numpy().tobytes()


def decode(bitstream: bytes, cdfs) -> np.ndarray:
    """One stream: bytes + CDFs [N, V+1] -> symbols [N] (one launch per symbol,
    as each symbol's CDF may depend on the previous one in real use)."""
    c = torch.as_tensor(np.asarray(cdfs).astype(np.int32) if isinstance(cdfs, np.ndarray) else cdfs)
    c = c.cuda().to(torch.int32).contiguous()
    n, vp1 = c.shape
    out = torch.empty(max(n, 1), dtype=torch.int32, device=c.device)
    if n == 0:
        return np.zeros(0, np.int32)
    bits = _bits_of(c)
    buf = torch.from_numpy(np.frombuffer(bytes(bitstream) + b"\0" * 64, np.uint8).copy()).cuda()
    st = torch.empty(4, dtype=torch.int32, device=c.device)
    sp = N.stream_ptr(c.device)
    N.call("kb_coder_decode_init", buf.data_ptr(), len(bitstream), None, st.data_ptr(), 1, sp)
    for i in range(n):
        N.call("kb_coder_decode_cdf", c[i].data_ptr(), vp1, vp1 - 1, bits, buf.data_ptr(),
               len(bitstream), None, st.data_ptr(), out[i:].data_ptr(), 1, sp)
    return out[:n].cpu().numpy()


def encode_chunk_gpu(probs_iter, symbols_iter, max_output_bytes: int,
                     bits: int = CDF_PRECISION) -> bytes:
    """Stream-encode a chunk batch by batch with persistent coder state."""
    out = st = None
    sp = None
    for probs, symbols in zip(probs_iter, symbols_iter):
        if out is None:
            dev = probs.device
            sp = N.stream_ptr(dev)
            out = torch.zeros(max_output_bytes, dtype=torch.uint8, device=dev)
            st = torch.empty(4, dtype=torch.int32, device=dev)
            N.call("kb_coder_encode_init", st.data_ptr(), 1, sp)
        cdf = probs_to_cdf_gpu(probs, bits)
        sym = symbols.to(torch.int32).contiguous()
        N.call("kb_coder_encode_cdf", cdf.data_ptr(), cdf.shape[1], sym.data_ptr(),
               cdf.shape[0], bits, out.data_ptr(), max_output_bytes, st.data_ptr(), sp)
    if out is None:
        return b""
    N.call("kb_coder_encode_finalize", out.data_ptr(), max_output_bytes, None, st.data_ptr(), 1, sp)
    nbytes = ((int(st[3].item()) & 0xFFFFFFFF) + 7) // 8
    if nbytes > max_output_bytes:
        raise RuntimeError("encoded stream exceeded max_output_bytes")
    return out[:nbytes].cpu().numpy().tobytes()
