"""The reference extension's function names over the krunch_b200 C ABI.

Same tensor contracts as krunch_ac/cuda/main.cpp:114-303 and
layer_cpp.cpp:728-849,1041-1052: CUDA tensors, contiguous, state tensors of
4 x uint32 per stream, base_byte_offsets int32, work enqueued on the current
stream without a sync.  CDF totals are 2^CDF_PRECISION (24, as
range_coder.cuh:19 hard-codes).  Every call runs a krunch_b200 kernel.
"""
from __future__ import annotations

import torch

from . import _native as N

CDF_PRECISION = 24


def _chk(t: torch.Tensor, name: str, dtypes) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")
    if t.dtype not in dtypes:
        raise RuntimeError(f"{name} has dtype {t.dtype}, expected one of {dtypes}")


_I32 = (torch.int32,)
_U32 = (torch.uint32, torch.int32)
_U8 = (torch.uint8,)


def _offs64(base_byte_offsets: torch.Tensor) -> torch.Tensor:
    _chk(base_byte_offsets, "base_byte_offsets", _I32 + (torch.int64,))
    return base_byte_offsets.to(torch.int64)


def encode_step(cdf, symbols, output_buf, state):
    _chk(cdf, "cdf", _I32), _chk(symbols, "symbols", _I32), _chk(output_buf, "output_buf", _U8)
    _chk(state, "state", _U32)
    if cdf.dim() != 2 or symbols.numel() != cdf.shape[0]:
        raise RuntimeError("cdf must be (N, V+1) with one symbol per row")
    N.call("kb_coder_encode_cdf", cdf.data_ptr(), cdf.shape[1], symbols.data_ptr(), cdf.shape[0],
           CDF_PRECISION, output_buf.data_ptr(), output_buf.numel(), state.data_ptr(),
           N.stream_ptr(cdf.device))


def encode_finalize(output_buf, state):
    _chk(output_buf, "output_buf", _U8), _chk(state, "state", _U32)
    N.call("kb_coder_encode_finalize", output_buf.data_ptr(), output_buf.numel(), None,
           state.data_ptr(), 1, N.stream_ptr(state.device))


def decode_init(input_buf, state):
    _chk(input_buf, "input_buf", _U8), _chk(state, "state", _U32)
    N.call("kb_coder_decode_init", input_buf.data_ptr(), input_buf.numel(), None, state.data_ptr(),
           1, N.stream_ptr(state.device))


def decode_step(cdf, input_buf, state, out_sym):
    _chk(cdf, "cdf", _I32), _chk(input_buf, "input_buf", _U8), _chk(state, "state", _U32)
    _chk(out_sym, "out_sym", _I32)
    V = cdf.numel() - 1
    N.call("kb_coder_decode_cdf", cdf.data_ptr(), V + 1, V, CDF_PRECISION, input_buf.data_ptr(),
           input_buf.numel(), None, state.data_ptr(), out_sym.data_ptr(), 1,
           N.stream_ptr(cdf.device))


def decode_init_batched(input_buf, base_byte_offsets, states):
    _chk(input_buf, "input_buf", _U8), _chk(states, "states", _U32)
    offs = _offs64(base_byte_offsets)
    N.call("kb_coder_decode_init", input_buf.data_ptr(), input_buf.numel(), offs.data_ptr(),
           states.data_ptr(), offs.numel(), N.stream_ptr(states.device))


def decode_step_batched(cdfs, input_buf, base_byte_offsets, states, out_syms):
    _chk(cdfs, "cdfs", _I32), _chk(input_buf, "input_buf", _U8), _chk(states, "states", _U32)
    _chk(out_syms, "out_syms", _I32)
    offs = _offs64(base_byte_offsets)
    B, vp1 = cdfs.shape
    N.call("kb_coder_decode_cdf", cdfs.data_ptr(), vp1, vp1 - 1, CDF_PRECISION,
           input_buf.data_ptr(), input_buf.numel(), offs.data_ptr(), states.data_ptr(),
           out_syms.data_ptr(), B, N.stream_ptr(cdfs.device))


def encode_step_batched(cdfs, symbols, output_buf, base_byte_offsets, states):
    _chk(cdfs, "cdfs", _I32), _chk(symbols, "symbols", _I32), _chk(output_buf, "output_buf", _U8)
    _chk(states, "states", _U32)
    offs = _offs64(base_byte_offsets)
    B, vp1 = cdfs.shape
    N.call("kb_coder_encode_cdf_batched", cdfs.data_ptr(), vp1, symbols.data_ptr(), B,
           CDF_PRECISION, output_buf.data_ptr(), output_buf.numel(), offs.data_ptr(),
           states.data_ptr(), N.stream_ptr(cdfs.device))


def encode_finalize_batched(output_buf, base_byte_offsets, states):
    _chk(output_buf, "output_buf", _U8), _chk(states, "states", _U32)
    offs = _offs64(base_byte_offsets)
    N.call("kb_coder_encode_finalize", output_buf.data_ptr(), output_buf.numel(), offs.data_ptr(),
           states.data_ptr(), offs.numel(), N.stream_ptr(states.device))


def det_softmax_cdf(logits: torch.Tensor, cdf_T: int) -> torch.Tensor:
    """fp16 logits [T, V] -> int32 [T, V+1]: 0 then the per-symbol counts
    (the caller cumsums, as the reference's binding does)."""
    _chk(logits, "logits", (torch.float16,))
    T = int(cdf_T)
    if T <= 0 or T & (T - 1):
        raise RuntimeError("cdf_T must be a power of two")
    rows, V = logits.shape
    out = torch.empty((rows, V + 1), dtype=torch.int32, device=logits.device)
    N.call("kb_cdf_rows", logits.data_ptr(), V, rows, V, T.bit_length() - 1, N.KB_CDF_COUNTS,
           None, 0, None, out.data_ptr(), N.stream_ptr(logits.device))
    return out


def det_matmul(x: torch.Tensor, W: torch.Tensor, out_dtype=None) -> torch.Tensor:
    """x f16 [M, K] @ W f16 [K, N] (reference [in, out] layout) with the
    M-invariant krunch_b200 GEMM; fp32 accumulation."""
    _chk(x, "x", (torch.float16,)), _chk(W, "W", (torch.float16,))
    M, K = x.shape
    K2, Nn = W.shape
    if K != K2:
        raise RuntimeError("inner dimensions differ")
    Kp, Np = (K + 63) // 64 * 64, (Nn + 127) // 128 * 128
    Wt = torch.zeros((Np, Kp), dtype=torch.float16, device=W.device)
    Wt[:Nn, :K] = W.t()
    xa = x if Kp == K else torch.nn.functional.pad(x, (0, Kp - K)).contiguous()
    f32 = out_dtype == torch.float32
    out = torch.empty((M, Np), dtype=torch.float32 if f32 else torch.float16, device=x.device)
    N.call("kb_gemm", N.KB_F16, xa.data_ptr(), Kp, Wt.data_ptr(), Kp, M, Np, Kp,
           N.KB_EPI_F32 if f32 else N.KB_EPI_F16, out.data_ptr(), Np, None, None,
           N.stream_ptr(x.device))
    return out[:, :Nn] if Np != Nn else out
