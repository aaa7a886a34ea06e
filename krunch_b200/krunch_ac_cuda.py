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


def _det_matmul(x: torch.Tensor, W: torch.Tensor, out_dtype, kind: int, dt) -> torch.Tensor:
    _chk(x, "x", (dt,)), _chk(W, "W", (dt,))
    M, K = x.shape
    K2, Nn = W.shape
    if K != K2:
        raise RuntimeError("inner dimensions differ")
    Kp, Np = (K + 63) // 64 * 64, (Nn + 127) // 128 * 128
    Wt = torch.zeros((Np, Kp), dtype=dt, device=W.device)
    Wt[:Nn, :K] = W.t()
    xa = x if Kp == K else torch.nn.functional.pad(x, (0, Kp - K)).contiguous()
    f32 = out_dtype == torch.float32
    out = torch.empty((M, Np), dtype=torch.float32 if f32 else torch.float16, device=x.device)
    N.call("kb_gemm", kind, xa.data_ptr(), Kp, Wt.data_ptr(), Kp, M, Np, Kp,
           N.KB_EPI_F32 if f32 else N.KB_EPI_F16, out.data_ptr(), Np, None, None,
           N.stream_ptr(x.device))
    out = out[:, :Nn] if Np != Nn else out
    if out_dtype is not None and out.dtype != out_dtype:
        out = out.to(out_dtype)
    return out


def det_matmul(x: torch.Tensor, W: torch.Tensor, out_dtype=None) -> torch.Tensor:
    """x f16 [M, K] @ W f16 [K, N] (reference [in, out] layout) with the
    M-invariant krunch_b200 GEMM; fp32 accumulation (layer_cpp.cpp:846-849)."""
    return _det_matmul(x, W, out_dtype, N.KB_F16, torch.float16)


def det_matmul_bf16(x: torch.Tensor, W: torch.Tensor, out_dtype=None) -> torch.Tensor:
    """bf16 x [M, K] @ bf16 W [K, N], fp32 accumulation; bf16 out unless
    out_dtype says otherwise (layer_cpp.cpp:850-870)."""
    # bf16 output (the reference's default: x's dtype) rounds once from fp32
    if out_dtype in (None, torch.bfloat16):
        return _det_matmul(x, W, torch.float32, N.KB_BF16, torch.bfloat16).to(torch.bfloat16)
    return _det_matmul(x, W, out_dtype, N.KB_BF16, torch.bfloat16)


def det_matmul_tc_3way_async(A0, A1, A2, B0, B1, B2, out_dtype=None):
    """(A0 @ B0, A1 @ B1, A2 @ B2) for inputs sharing [M, K] and weights
    sharing [K, N] (layer_cpp.cpp:926-960): plain products in one dtype, as
    the reference's binding returns them."""
    for a in (A1, A2):
        if a.shape != A0.shape:
            raise RuntimeError("M must match")
    for b in (B1, B2):
        if b.shape[-1] != B0.shape[-1]:
            raise RuntimeError("N must match")
    return tuple(det_matmul(a, b, out_dtype) for a, b in zip((A0, A1, A2), (B0, B1, B2)))


def reset_phase_times() -> None:
    """Start accumulating per-phase device times (the reference's
    KRUNCH_PHASE_PROFILE accumulators, layer_cpp.cpp:833-837): every library
    launch until read_phase_times() is bracketed by CUDA events."""
    N.profile_begin()


def read_phase_times() -> dict:
    """Milliseconds per phase since reset_phase_times(), plus call_count (the
    launches counted); the phases are this library's (embed, ln_mix, gemm,
    wkv, head, cdf, encode, decode, step).  Like the reference's, meant for
    a single host thread; reading ends the accumulation."""
    prof = N.profile_end()
    d = {k: v[0] for k, v in prof.items()}
    d["call_count"] = int(sum(v[1] for v in prof.values()))
    return d


# --------------------------------------------------------------------------
# rwkv4_layer_step_cpp / rwkv4_layer_step_cpp_t1 (layer_cpp.cpp:294-307,
# 456-637): one RWKV-4 layer over x [B, T, C] with the 18 layer tensors in
# the order of cpp_path.init_weights (cpp_path.py:59-78) — LN and mixes
# fp16 [C], time_decay / time_first fp32 [C] as the rwkv loader leaves them
# (time_decay already -exp(raw)), matrices [in, out] fp16 (or bf16).  The
# layer runs the production WKV convention, as the reference's layer does
# (rwkv::wkv_forward or its own wkv_kernel.cu:57-72).  State tensors
# att_xx / ffn_xx [B, C] (fp16), aa / bb / pp [B, C] fp32 are updated in
# place; the new x is returned.
# --------------------------------------------------------------------------

class _LayerHandle:
    """A one-layer kb_model over device copies of the reference's layer
    tensors in this library's layout (matrices K-major, LN / mixes fp32,
    decay = -time_decay).  Cached per set of input tensors, like the
    reference's weight and graph caches (one host thread per process)."""

    def __init__(self, w, dev):
        import ctypes as C
        (ln1_w, ln1_b, tm_k, tm_v, tm_r, td, tf, Kw, Vw, Rw, Ow,
         ln2_w, ln2_b, ftm_k, ftm_r, fKw, fVw, fRw) = w
        self.keep = []
        Cm = Kw.shape[0]
        Fm = fKw.shape[1]
        bf = Kw.dtype == torch.bfloat16
        for t, nm in ((Kw, "Kw"), (Vw, "Vw"), (Rw, "Rw"), (Ow, "Ow"), (fKw, "ffn_Kw"),
                      (fVw, "ffn_Vw"), (fRw, "ffn_Rw")):
            if t.dtype not in (torch.float16, torch.bfloat16) or t.dtype != Kw.dtype:
                raise RuntimeError(f"{nm} must be fp16 or bf16 like Kw")
        if tuple(Kw.shape) != (Cm, Cm) or tuple(fVw.shape) != (Fm, Cm):
            raise RuntimeError("layer matrices must be [in, out] with n_att == n_embd")

        def f32(t):
            t = t.detach().reshape(-1).to(dev, torch.float32).contiguous()
            self.keep.append(t)
            return t.data_ptr()

        def km(t):
            t = t.detach().to(dev).t().contiguous()
            self.keep.append(t)
            return t.data_ptr()

        d = N.LayerDesc()
        d.ln1_w, d.ln1_b, d.ln2_w, d.ln2_b = f32(ln1_w), f32(ln1_b), f32(ln2_w), f32(ln2_b)
        d.att_mix_k, d.att_mix_v, d.att_mix_r = f32(tm_k), f32(tm_v), f32(tm_r)
        d.att_decay = f32(-td.float())
        d.att_first = f32(tf)
        d.att_kw, d.att_vw, d.att_rw, d.att_ow = km(Kw), km(Vw), km(Rw), km(Ow)
        d.ffn_mix_k, d.ffn_mix_r = f32(ftm_k), f32(ftm_r)
        d.ffn_kw, d.ffn_vw, d.ffn_rw = km(fKw), km(fVw), km(fRw)
        self.layers = (N.LayerDesc * 1)(d)
        # the layer entry never reads the embedding, final LayerNorm or head:
        # a 128-row placeholder satisfies the model description
        dummy = torch.zeros((128, Cm), dtype=Kw.dtype, device=dev)
        ones = torch.ones(Cm, dtype=torch.float32, device=dev)
        self.keep += [dummy, ones]
        md = N.ModelDesc()
        md.n_layer, md.n_embd, md.n_ffn, md.n_vocab, md.vocab_pad = 1, Cm, Fm, 128, 128
        md.wdtype = N.KB_BF16 if bf else N.KB_F16
        md.wkv_convention = N.KB_WKV_PRODUCTION
        md.emb, md.head = dummy.data_ptr(), dummy.data_ptr()
        md.ln_out_w = md.ln_out_b = ones.data_ptr()
        md.layers = self.layers
        md.head_scale = None
        h = C.c_void_p()
        N.call("kb_model_create", C.byref(md), C.byref(h))
        self.handle = h
        self.C, self.F = Cm, Fm
        self.ws = None

    def workspace(self, B, T, dev):
        n = int(N.load().kb_forward_workspace_bytes(self.handle, B, T))
        if self.ws is None or self.ws.numel() < n:
            self.ws = torch.empty(n, dtype=torch.uint8, device=dev)
        return self.ws

    def __del__(self):
        h = getattr(self, "handle", None)
        if h is not None and h.value:
            try:
                N.load().kb_model_destroy(h)
            except Exception:
                pass


_LAYER_CACHE: dict = {}


def _layer_handle(w, dev) -> _LayerHandle:
    """The converted layer for these 18 tensors.  The entry holds the source
    tensors, so their addresses cannot be reused by other tensors while it
    is cached, and the key includes each tensor's in-place version counter,
    so an edited tensor is converted again."""
    key = tuple((t.data_ptr(), tuple(t.shape), t.dtype, t._version) for t in w)
    h = _LAYER_CACHE.get(key)
    if h is None:
        h = _LAYER_CACHE[key] = _LayerHandle(w, dev)
        h.src = tuple(w)
    return h


def clear_layer_graph_cache() -> None:
    """Drop the cached layer handles and the tensors they hold (the
    reference's cache reset, layer_cpp.cpp:1038)."""
    _LAYER_CACHE.clear()


def rwkv4_layer_step_cpp(x, att_xx, aa, bb, pp, ffn_xx, *layer):
    if len(layer) != 18:
        raise RuntimeError(f"expected 18 layer tensors, got {len(layer)}")
    _chk(x, "x", (torch.float16,))
    if x.dim() != 3:
        raise RuntimeError("x must be [B, T, C]")
    B, T, Cm = x.shape
    for t, nm in ((aa, "aa"), (bb, "bb"), (pp, "pp")):
        _chk(t, nm, (torch.float32,))
    for t, nm in ((att_xx, "att_xx"), (ffn_xx, "ffn_xx")):
        _chk(t, nm, (torch.float16, torch.bfloat16, torch.float32))
    for t, nm in zip((att_xx, aa, bb, pp, ffn_xx), ("att_xx", "aa", "bb", "pp", "ffn_xx")):
        if t.numel() != B * Cm:
            raise RuntimeError(f"{nm} must hold [B, C] = [{B}, {Cm}]")
    h = _layer_handle(layer, x.device)
    if h.C != Cm:
        raise RuntimeError("x width differs from the layer's n_embd")
    st = torch.stack([t.reshape(B, Cm).float() for t in (att_xx, aa, bb, pp, ffn_xx)]).contiguous()
    out = x.reshape(B * T, Cm).clone()
    ws = h.workspace(B, T, x.device)
    N.call("kb_layer_forward", h.handle, 0, out.data_ptr(), B, T, st.data_ptr(), ws.data_ptr(),
           ws.numel(), N.stream_ptr(x.device))
    for i, t in enumerate((att_xx, aa, bb, pp, ffn_xx)):
        t.copy_(st[i].view_as(t))
    return out.view(B, T, Cm)


def rwkv4_layer_step_cpp_t1(x, att_xx, aa, bb, pp, ffn_xx, *layer):
    """The single-token form ([1, 1, C]); the same kernels as any window."""
    if x.dim() != 3 or x.shape[0] != 1 or x.shape[1] != 1:
        raise RuntimeError("x must be [1, 1, C]")
    return rwkv4_layer_step_cpp(x, att_xx, aa, bb, pp, ffn_xx, *layer)
