"""Batched RWKV-4 forward with the reference's call shape and state contract
(krunch/batched_rwkv4.py:60-82 init_state_batched, 175-262 forward_batched).

``m`` is a krunch_b200.model.RWKVModel.  The state is the reference's list of
5 * n_layer tensors: per layer i

    5i+0 att_xx [B, C] activation dtype (fp16; bf16 for a bf16 model)
    5i+1 aa     [B, C] fp32
    5i+2 bb     [B, C] fp32
    5i+3 pp     [B, C] fp32, -1e30 initially
    5i+4 ffn_xx [B, C] activation dtype

``forward_batched`` rebinds the list's entries to the advanced state (the
reference assigns ``state[i*5+s] = ...`` in place of the list it was given),
and returns it.  The kernels keep the state as one fp32 [n_layer, 5, B, C]
tensor; att_xx / ffn_xx hold LayerNorm outputs rounded to the activation
dtype, so the conversion in both directions is exact.  A stacked tensor from
``RWKVModel.new_state`` is accepted as well and advanced in place.

Logits come back in the activation dtype, as the reference's
``x @ w['head.weight']`` does: [B, T, V] (or [B, V] with full_output False),
a view of the kernel's padded head output (no copy).
"""
from __future__ import annotations

import torch

from .model import RWKVModel


def _atype(m: RWKVModel) -> torch.dtype:
    return torch.bfloat16 if m.spec.wdtype == "bf16" else torch.float16


def init_state_batched(m: RWKVModel, B: int, device=None) -> list[torch.Tensor]:
    """Fresh state list (krunch/batched_rwkv4.py:60-82)."""
    s = m.spec
    dev = m.device if device is None else torch.device(device)
    at = _atype(m)
    st: list[torch.Tensor] = []
    for _ in range(s.n_layer):
        st.append(torch.zeros((B, s.n_embd), dtype=at, device=dev))
        st.append(torch.zeros((B, s.n_embd), dtype=torch.float32, device=dev))
        st.append(torch.zeros((B, s.n_embd), dtype=torch.float32, device=dev))
        st.append(torch.full((B, s.n_embd), -1e30, dtype=torch.float32, device=dev))
        st.append(torch.zeros((B, s.n_embd), dtype=at, device=dev))
    return st


def state_list(state: torch.Tensor, atype: torch.dtype | None = None) -> list[torch.Tensor]:
    """Stacked fp32 [L, 5, B, C] -> the reference's 5*L list (att_xx /
    ffn_xx converted to ``atype`` when given, else views)."""
    out = []
    for i in range(state.shape[0]):
        for s in range(5):
            t = state[i, s]
            if atype is not None and s in (0, 4):
                t = t.to(atype)
            out.append(t)
    return out


def state_from_list(lst: list[torch.Tensor]) -> torch.Tensor:
    """The reference's 5*L list -> stacked fp32 [L, 5, B, C]."""
    L = len(lst) // 5
    return torch.stack([torch.stack([lst[5 * i + s].float() for s in range(5)])
                        for i in range(L)]).contiguous()


def forward_batched(m: RWKVModel, tokens_batches, state=None, full_output: bool = True):
    """tokens [B, T] (list of equal-length token lists, or a tensor; a 1-D
    tensor is [B] single tokens) -> (logits, state)."""
    if isinstance(tokens_batches, torch.Tensor):
        idx = tokens_batches
        if idx.dim() == 1:
            idx = idx.unsqueeze(1)
    else:
        B = len(tokens_batches)
        T = len(tokens_batches[0])
        if any(len(b) != T for b in tokens_batches):
            raise AssertionError("all batch streams must have same token-length T (caller pads)")
        idx = torch.as_tensor(tokens_batches)
    idx = idx.to(device=m.device, dtype=torch.int32).contiguous()
    B, T = idx.shape
    if state is None:
        state = init_state_batched(m, B)
    if isinstance(state, torch.Tensor):
        stacked, as_list = state, None
    else:
        if len(state) != 5 * m.spec.n_layer:
            raise ValueError(f"state must hold {5 * m.spec.n_layer} tensors, got {len(state)}")
        stacked, as_list = state_from_list([t.to(m.device) for t in state]), state
    ws = m.new_workspace(B, T)
    logits = m.new_logits(B, T)
    m.forward_window(idx, stacked, ws, logits)
    V = m.spec.n_vocab
    out = logits.view(B, T, -1)[:, :, :V]
    if _atype(m) != out.dtype:
        out = out.to(_atype(m))
    if not full_output:
        out = out[:, -1, :]
    if as_list is not None:
        at = _atype(m)
        for i, t in enumerate(state_list(stacked)):
            as_list[i] = t.to(at) if i % 5 in (0, 4) else t.clone()
        return out, as_list
    return out, stacked
