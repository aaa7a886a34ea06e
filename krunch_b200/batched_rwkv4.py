"""Batched RWKV-4 forward with the reference's call shape
(krunch/batched_rwkv4.py:60-82 init_state_batched, 175-262 forward_batched).

``m`` is a krunch_b200.model.RWKVModel.  State is the model's fp32
[n_layer, 5, B, C] tensor (the reference's 5-per-layer list, stacked);
``state_list`` / ``state_from_list`` convert between the two.
"""
from __future__ import annotations

import torch

from .model import RWKVModel


def init_state_batched(m: RWKVModel, B: int, device=None) -> torch.Tensor:
    return m.new_state(B)


def state_list(state: torch.Tensor) -> list[torch.Tensor]:
    L = state.shape[0]
    return [state[i, s] for i in range(L) for s in range(5)]


def state_from_list(lst: list[torch.Tensor]) -> torch.Tensor:
    L = len(lst) // 5
    return torch.stack([torch.stack([lst[5 * i + s].float() for s in range(5)])
                        for i in range(L)]).contiguous()


def forward_batched(m: RWKVModel, tokens_batches, state: torch.Tensor | None = None,
                    full_output: bool = True):
    """tokens [B, T] (list of equal-length lists or a tensor) -> (logits, state).

    logits: fp32 [B, T, V] (or [B, V] when full_output is False); the state
    is advanced in place and returned."""
    if isinstance(tokens_batches, torch.Tensor):
        idx = tokens_batches
        if idx.dim() == 1:
            idx = idx.unsqueeze(1)
    else:
        idx = torch.as_tensor(tokens_batches)
    idx = idx.to(device=m.device, dtype=torch.int32).contiguous()
    B, T = idx.shape
    if state is None:
        state = m.new_state(B)
    ws = m.new_workspace(B, T)
    logits = m.new_logits(B, T)
    m.forward_window(idx, state, ws, logits)
    V = m.spec.n_vocab
    out = logits[:, :V].float().view(B, T, V)
    if not full_output:
        out = out[:, -1, :]
    return out, state
