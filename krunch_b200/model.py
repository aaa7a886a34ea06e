"""RWKV-4 model resident on one B200: device weights + the native model handle.

Replaces krunch/cpp_path.py:init_weights / fresh_state (cpp_path.py:26-106).
Weights arrive in the reference's ``model.w`` layout (matrices [in, out],
time_decay as the raw log-decay of rwkv4_step_ref.py:89) and are stored on
the device K-major ([out, in], fp16) for the GEMMs.

``wdtype="bf16"`` keeps every matrix in bf16 and feeds the GEMMs bf16
inputs (the reference's KRUNCH_BF16 route, krunch_ac/cuda/layer_cpp.cpp:
224-241: activations otherwise fp16).  ``wdtype="i8"`` is the w8a8 model: every matrix (head included) quantised
per output channel to int8 with fp16 factors (kb_quantize_weight), the GEMM
inputs quantised per row at run time.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from . import _native as N


@dataclass(frozen=True)
class ModelSpec:
    n_layer: int
    n_embd: int
    n_ffn: int
    n_vocab: int
    wdtype: str = "f16"
    wkv: str = "step_ref"

    @property
    def vocab_pad(self) -> int:
        return (self.n_vocab + 127) // 128 * 128


def _n_layer(w: dict) -> int:
    n = 0
    while f"blocks.{n}.ln1.weight" in w:
        n += 1
    return n


class RWKVModel:
    """Device-resident RWKV-4 with a kb_model handle."""

    def __init__(self, w: dict, device="cuda", wkv: str = "step_ref", wdtype: str = "f16"):
        if wdtype not in ("f16", "bf16", "i8"):
            raise ValueError(f"unknown weight dtype {wdtype!r}")
        if wkv not in ("step_ref", "production"):
            raise ValueError(f"unknown WKV convention {wkv!r}")
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("krunch_b200 runs on CUDA devices only")
        L = _n_layer(w)
        V, Cm = w["emb.weight"].shape
        F = w["blocks.0.ffn.key.weight"].shape[1]
        self.spec = ModelSpec(L, Cm, F, V, wdtype, wkv)
        self._keep: list[torch.Tensor] = []
        dev = self.device

        def f32(a):
            t = torch.as_tensor(np.ascontiguousarray(a, dtype=np.float32).reshape(-1)).to(dev)
            self._keep.append(t)
            return t

        stream = N.stream_ptr(dev)
        i8 = wdtype == "i8"

        def quantize(t16):  # fp16 [N, K] -> (int8 [N, K], fp16 scales [N])
            q = torch.empty(t16.shape, dtype=torch.int8, device=dev)
            sc = torch.empty(t16.shape[0], dtype=torch.float16, device=dev)
            N.call("kb_quantize_weight", t16.data_ptr(), t16.shape[0], t16.shape[1], q.data_ptr(),
                   sc.data_ptr(), stream)
            self._keep += [q, sc]
            return q, sc

        def kmajor(a):  # [in, out] -> fp16 [out, in]  (int8 + scales for i8, bf16 for bf16)
            t = torch.as_tensor(np.asarray(a, dtype=np.float32)).to(dev)
            if wdtype == "bf16":
                t = t.t().contiguous().to(torch.bfloat16)
                self._keep.append(t)
                return t, None
            t = t.t().contiguous().to(torch.float16)
            if i8:
                return quantize(t)
            self._keep.append(t)
            return t, None

        def mat(d, name, arr):
            q, sc = kmajor(arr)
            setattr(d, name + "w", q.data_ptr())
            if sc is not None:
                setattr(d, name + "s", sc.data_ptr())

        self.emb = torch.as_tensor(np.asarray(w["emb.weight"], np.float32)).to(dev).half().contiguous()
        self._keep.append(self.emb)
        layers = (N.LayerDesc * L)()
        for i in range(L):
            b, att, ffn = f"blocks.{i}.", f"blocks.{i}.att.", f"blocks.{i}.ffn."
            td = f32(w[att + "time_decay"])
            decay = torch.empty_like(td)
            self._keep.append(decay)
            N.call("kb_prepare_decay", td.data_ptr(), decay.data_ptr(), td.numel(), stream)
            d = layers[i]
            d.ln1_w, d.ln1_b = f32(w[b + "ln1.weight"]).data_ptr(), f32(w[b + "ln1.bias"]).data_ptr()
            d.ln2_w, d.ln2_b = f32(w[b + "ln2.weight"]).data_ptr(), f32(w[b + "ln2.bias"]).data_ptr()
            d.att_mix_k = f32(w[att + "time_mix_k"]).data_ptr()
            d.att_mix_v = f32(w[att + "time_mix_v"]).data_ptr()
            d.att_mix_r = f32(w[att + "time_mix_r"]).data_ptr()
            d.att_decay = decay.data_ptr()
            d.att_first = f32(w[att + "time_first"]).data_ptr()
            mat(d, "att_k", w[att + "key.weight"])
            mat(d, "att_v", w[att + "value.weight"])
            mat(d, "att_r", w[att + "receptance.weight"])
            mat(d, "att_o", w[att + "output.weight"])
            d.ffn_mix_k = f32(w[ffn + "time_mix_k"]).data_ptr()
            d.ffn_mix_r = f32(w[ffn + "time_mix_r"]).data_ptr()
            mat(d, "ffn_k", w[ffn + "key.weight"])
            mat(d, "ffn_v", w[ffn + "value.weight"])
            mat(d, "ffn_r", w[ffn + "receptance.weight"])
        Vp = self.spec.vocab_pad
        hdt = torch.bfloat16 if wdtype == "bf16" else torch.float16
        head = torch.zeros((Vp, Cm), dtype=hdt, device=dev)
        head[:V] = torch.as_tensor(np.asarray(w["head.weight"], np.float32)).to(dev).t().to(hdt)
        self.head_scale = None
        if i8:
            head, self.head_scale = quantize(head)
        else:
            self._keep.append(head)
        self.head = head
        self._layers = layers
        desc = N.ModelDesc()
        desc.n_layer, desc.n_embd, desc.n_ffn, desc.n_vocab = L, Cm, F, V
        desc.vocab_pad = Vp
        desc.wdtype = {"f16": N.KB_F16, "bf16": N.KB_BF16, "i8": N.KB_I8}[wdtype]
        desc.wkv_convention = N.KB_WKV_STEP_REF if wkv == "step_ref" else N.KB_WKV_PRODUCTION
        desc.emb = self.emb.data_ptr()
        desc.ln_out_w = f32(w["ln_out.weight"]).data_ptr()
        desc.ln_out_b = f32(w["ln_out.bias"]).data_ptr()
        desc.head = head.data_ptr()
        desc.layers = layers
        desc.head_scale = None if self.head_scale is None else self.head_scale.data_ptr()
        handle = C.c_void_p()
        N.call("kb_model_create", C.byref(desc), C.byref(handle))
        self.handle = handle
        torch.cuda.synchronize(dev)

    def __del__(self):
        h = getattr(self, "handle", None)
        if h is not None and h.value:
            try:
                N.load().kb_model_destroy(h)
            except Exception:
                pass
            self.handle = None

    # ------------------------------------------------------------------ state
    def state_numel(self, B: int) -> int:
        s = self.spec
        return s.n_layer * 5 * B * s.n_embd

    def new_state(self, B: int) -> torch.Tensor:
        """fp32 [n_layer, 5, B, C]: att_xx, aa, bb, pp (-1e30), ffn_xx."""
        s = self.spec
        st = torch.empty((s.n_layer, 5, B, s.n_embd), dtype=torch.float32, device=self.device)
        N.call("kb_state_init", self.handle, st.data_ptr(), B, N.stream_ptr(self.device))
        return st

    # ---------------------------------------------------------------- forward
    def workspace_bytes(self, B: int, T: int) -> int:
        return int(N.load().kb_forward_workspace_bytes(self.handle, B, T))

    def new_workspace(self, B: int, T: int) -> torch.Tensor:
        return torch.empty(self.workspace_bytes(B, T), dtype=torch.uint8, device=self.device)

    def new_logits(self, B: int, T: int) -> torch.Tensor:
        return torch.empty((B * T, self.spec.vocab_pad), dtype=torch.float16, device=self.device)

    @property
    def stats_stride(self) -> int:
        """Softmax partials per logits row (one per 32 head columns)."""
        return self.spec.vocab_pad // 32

    def new_stats(self, B: int, T: int) -> torch.Tensor:
        return torch.empty((B * T, self.stats_stride, 2), dtype=torch.float32, device=self.device)

    # ------------------------------------------------------ fused decode step
    @property
    def has_fused_step(self) -> bool:
        """The w8a8 model (up to C = 768) decodes through kb_step_forward (one
        persistent launch for the layer stack)."""
        # measured: at C = 2048 (1.5B, B = 512) the per-op chain is faster
        # (4.96 vs 7.09 ms/step); at C = 768 the fused step is (0.60 vs 1.09)
        return self.spec.wdtype == "i8" and self.spec.n_embd <= 768

    def new_step_workspace(self, B: int) -> torch.Tensor:
        n = int(N.load().kb_step_workspace_bytes(self.handle, B))
        return torch.empty(n, dtype=torch.uint8, device=self.device)

    def step_forward(self, tokens: torch.Tensor, state: torch.Tensor, workspace: torch.Tensor,
                     logits: torch.Tensor, stats: torch.Tensor | None = None) -> torch.Tensor:
        """forward_window for T = 1 through the fused step kernel (w8a8
        models): the same bits as forward_window(tokens[:, None], ...)."""
        B = tokens.shape[0]
        assert tokens.dtype == torch.int32 and tokens.is_contiguous()
        assert state.is_contiguous() and state.numel() == self.state_numel(B)
        N.call("kb_step_forward", self.handle, tokens.data_ptr(), B, state.data_ptr(),
               workspace.data_ptr(), workspace.numel(), logits.data_ptr(),
               None if stats is None else stats.data_ptr(), N.stream_ptr(self.device))
        return logits

    def forward_window(self, tokens: torch.Tensor, state: torch.Tensor, workspace: torch.Tensor,
                       logits: torch.Tensor, stats: torch.Tensor | None = None) -> torch.Tensor:
        """tokens int32 [B, T] (contiguous, on device) -> logits fp16 [B*T, vocab_pad].

        ``state`` is read and advanced in place.  With ``stats`` (from
        new_stats) the head writes, instead of raw logits, the per-32-column
        softmax numerators into ``logits`` and their partials into ``stats``
        (the input kb_cdf_rows / kb_decode_logits_step take)."""
        B, T = tokens.shape
        assert tokens.dtype == torch.int32 and tokens.is_contiguous()
        assert state.is_contiguous() and state.numel() == self.state_numel(B)
        assert logits.shape[0] >= B * T and logits.shape[1] == self.spec.vocab_pad
        N.call("kb_forward_window", self.handle, tokens.data_ptr(), B, T, state.data_ptr(),
               workspace.data_ptr(), workspace.numel(), logits.data_ptr(),
               None if stats is None else stats.data_ptr(), N.stream_ptr(self.device))
        return logits
