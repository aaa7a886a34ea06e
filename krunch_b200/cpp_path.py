"""The reference's bit-exact orchestration API (krunch/cpp_path.py) over this
build's kernels.

Same names and contracts as the reference:

* ``init_weights(model)`` — ``model`` is anything with the reference's
  ``model.w`` dict (an ``rwkv.model.RWKV``, or a namespace holding ``w``), or
  the dict itself; returns the device-resident ``RWKVModel`` (cached by id,
  cpp_path.py:26-91).  ``KRUNCH_BF16=1`` selects bf16 matrices, as there.
* ``fresh_state`` / ``fresh_state_batched`` — the 5-tuple of per-layer lists
  (att_xx fp16, aa / bb fp32, pp fp32 at -1e30, ffn_xx fp16), each entry
  [B, C] (cpp_path.py:94-106, 412-425).
* ``forward_packed`` / ``forward_packed_window`` / ``forward_stepped_batched``
  / ``forward_stepped`` — logits fp16, state mutated in place
  (cpp_path.py:109-163, 428-487).
* ``softmax_cdfs_per_row`` / ``softmax_cdf_one_row`` — int32 CDFs at the
  krunch_ac total 2^CDF_PRECISION (cpp_path.py:490-512).
* ``compute_decompress_batch`` (cpp_path.py:531-580).

The weights dict is the reference's ``model.w`` layout with raw
``time_decay`` (rwkv4_step_ref.py's convention); a loaded rwkv model whose
``time_decay`` already holds ``-exp(raw)`` is recognised by its sign (every
entry negative and ``model.version`` set) and converted back.  The forward
runs the step_ref WKV convention unless ``KRUNCH_WKV=production``.
"""
from __future__ import annotations

import os

import numpy as np
import torch

from . import _native as N
from .codec import compute_decompress_batch  # noqa: F401  (reference name)
from .model import RWKVModel

_WEIGHTS_CACHE: dict[int, RWKVModel] = {}


def _np(a):
    if isinstance(a, torch.Tensor):
        return a.detach().float().cpu().numpy()
    return np.asarray(a, dtype=np.float32)


def init_weights(model, device: str = "cuda") -> RWKVModel:
    key = id(model)
    if key in _WEIGHTS_CACHE:
        return _WEIGHTS_CACHE[key]
    w = model if isinstance(model, dict) else model.w
    loaded = not isinstance(model, dict) and getattr(model, "version", None) is not None
    wd = {}
    for k, v in w.items():
        a = _np(v)
        if k.endswith("time_decay") and loaded and (a < 0).all():
            a = np.log(-a)  # rwkv loader keeps -exp(raw)
        if k.endswith(("time_mix_k", "time_mix_v", "time_mix_r")):
            a = a.reshape(-1)
        wd[k] = a
    wdtype = "bf16" if os.environ.get("KRUNCH_BF16") == "1" else "f16"
    wkv = "production" if os.environ.get("KRUNCH_WKV") == "production" else "step_ref"
    m = RWKVModel(wd, device=device, wkv=wkv, wdtype=wdtype)
    _WEIGHTS_CACHE[key] = m
    return m


def _fresh(m: RWKVModel, B: int):
    s = m.spec
    dev = m.device
    at = torch.bfloat16 if s.wdtype == "bf16" else torch.float16
    L, C = s.n_layer, s.n_embd
    return ([torch.zeros(B, C, dtype=at, device=dev) for _ in range(L)],
            [torch.zeros(B, C, dtype=torch.float32, device=dev) for _ in range(L)],
            [torch.zeros(B, C, dtype=torch.float32, device=dev) for _ in range(L)],
            [torch.full((B, C), -1e30, dtype=torch.float32, device=dev) for _ in range(L)],
            [torch.zeros(B, C, dtype=at, device=dev) for _ in range(L)])


def fresh_state(weights: RWKVModel):
    return _fresh(weights, 1)


def fresh_state_batched(weights: RWKVModel, B: int):
    return _fresh(weights, B)


def _stack(state) -> torch.Tensor:
    L = len(state[0])
    return torch.stack([torch.stack([state[s][i].float() for s in range(5)])
                        for i in range(L)]).contiguous()


def _unstack(st: torch.Tensor, state) -> None:
    for i in range(st.shape[0]):
        for s in range(5):
            state[s][i].copy_(st[i, s].view_as(state[s][i]))


def _run(m: RWKVModel, ids: torch.Tensor, state, B: int, T: int) -> torch.Tensor:
    ids = ids.to(device=m.device, dtype=torch.int32).reshape(B, T).contiguous()
    st = _stack(state)
    logits = m.new_logits(B, T)
    m.forward_window(ids, st, m.new_workspace(B, T), logits)
    _unstack(st, state)
    return logits[:, :m.spec.n_vocab]


def forward_packed_window(weights: RWKVModel, input_ids, state, off: int, n: int) -> torch.Tensor:
    """Window [off, off+n) of one stream -> logits [n, V] fp16; windows
    compose exactly (state carried in place)."""
    if not isinstance(input_ids, torch.Tensor):
        input_ids = torch.as_tensor(input_ids, dtype=torch.long)
    ids = input_ids[off:off + n]
    return _run(weights, ids, state, 1, int(ids.shape[0]))


def forward_packed(weights: RWKVModel, input_ids, state) -> torch.Tensor:
    n = len(input_ids)
    return forward_packed_window(weights, input_ids, state, 0, n)


def forward_stepped_batched(weights: RWKVModel, last_tokens, state) -> torch.Tensor:
    """[B] previous tokens -> logits [B, V]; bit-identical per stream to
    forward_stepped and to the packed window."""
    if not isinstance(last_tokens, torch.Tensor):
        last_tokens = torch.as_tensor(last_tokens, dtype=torch.long)
    B = int(last_tokens.shape[0])
    return _run(weights, last_tokens, state, B, 1)


def forward_stepped(weights: RWKVModel, last_token: int, state) -> torch.Tensor:
    return _run(weights, torch.tensor([int(last_token)]), state, 1, 1).reshape(-1)


def softmax_cdfs_per_row(logits_TxV: torch.Tensor) -> torch.Tensor:
    """fp16 logits [T, V] -> int32 CDF [T, V+1] (fixed-order, row-local,
    bit-identical for any T)."""
    from .krunch_ac.cdf import CDF_PRECISION
    x = logits_TxV.to(torch.float16).contiguous()
    rows, V = x.shape
    out = torch.empty((rows, V + 1), dtype=torch.int32, device=x.device)
    N.call("kb_cdf_rows", x.data_ptr(), V, rows, V, CDF_PRECISION, N.KB_CDF_CDF, None, 0, None,
           out.data_ptr(), N.stream_ptr(x.device))
    return out


def softmax_cdf_one_row(logits_V: torch.Tensor) -> torch.Tensor:
    return softmax_cdfs_per_row(logits_V.reshape(1, -1))[0]
