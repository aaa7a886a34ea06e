"""RWKV-4 forward in numpy fp32 — TEST INFRASTRUCTURE ONLY.

Restates scripts/rwkv4_step_ref.py:41-165 (one token) and the packed form of
krunch/batched_rwkv4.py:85-262 with KRUNCH_PURE_WKV=1 (a window of T tokens
for B streams) on the reference's ``model.w`` layout (matrices [in, out]).

State: list of 5 * n_layer fp32 arrays [B, C] — att_xx, aa, bb, pp (init
-1e30), ffn_xx — the contract of init_state_batched (batched_rwkv4.py:60-82).
WKV conventions: "step_ref" (rwkv4_step_ref.py:76-94, the default) and
"production" (krunch_ac/cuda/wkv_kernel.cu:57-72, time_first on the key).
"""
from __future__ import annotations

import numpy as np


def n_layer_of(w: dict) -> int:
    n = 0
    while f"blocks.{n}.ln1.weight" in w:
        n += 1
    return n


def init_state(w: dict, B: int) -> list[np.ndarray]:
    L = n_layer_of(w)
    C = w["emb.weight"].shape[1]
    st = []
    for _ in range(L):
        st += [np.zeros((B, C), np.float32), np.zeros((B, C), np.float32),
               np.zeros((B, C), np.float32), np.full((B, C), -1e30, np.float32),
               np.zeros((B, C), np.float32)]
    return st


def layer_norm(x: np.ndarray, g: np.ndarray, b: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    m = x.mean(axis=-1, keepdims=True, dtype=np.float32)
    d = x - m
    var = (d * d).mean(axis=-1, keepdims=True, dtype=np.float32)
    return (d / np.sqrt(var + np.float32(eps)) * g + b).astype(np.float32)


def _sigmoid(x):
    return (1.0 / (1.0 + np.exp(-x))).astype(np.float32)


def _shift(xx: np.ndarray, prev: np.ndarray) -> np.ndarray:
    """[B,T,C] -> previous-token inputs (state for t=0)."""
    return np.concatenate([prev[:, None, :], xx[:, :-1, :]], axis=1)


def _mm(x: np.ndarray, W: np.ndarray) -> np.ndarray:
    B, T, C = x.shape
    return (x.reshape(B * T, C) @ W).reshape(B, T, W.shape[1])


def forward(w: dict, tokens: np.ndarray, state: list[np.ndarray] | None = None,
            wkv: str = "step_ref") -> tuple[np.ndarray, list[np.ndarray]]:
    """tokens int [B, T] -> (logits fp32 [B, T, V], new state)."""
    tok = np.asarray(tokens)
    if tok.ndim == 1:
        tok = tok[None]
    B, T = tok.shape
    if state is None:
        state = init_state(w, B)
    state = [s.copy() for s in state]
    x = w["emb.weight"][tok].astype(np.float32)
    for i in range(n_layer_of(w)):
        b, att, ffn = f"blocks.{i}.", f"blocks.{i}.att.", f"blocks.{i}.ffn."
        s = state[5 * i:5 * i + 5]
        xx = layer_norm(x, w[b + "ln1.weight"], w[b + "ln1.bias"])
        sx = _shift(xx, s[0])
        mk, mv, mr = (w[att + n].reshape(-1) for n in ("time_mix_k", "time_mix_v", "time_mix_r"))
        kx = xx * mk + sx * (1 - mk)
        vx = xx * mv + sx * (1 - mv)
        rx = xx * mr + sx * (1 - mr)
        r = _sigmoid(_mm(rx, w[att + "receptance.weight"]))
        k = _mm(kx, w[att + "key.weight"])
        v = _mm(vx, w[att + "value.weight"])
        u = w[att + "time_first"].reshape(-1)
        decay = np.exp(w[att + "time_decay"].reshape(-1)).astype(np.float32)
        aa, bb, pp = s[1], s[2], s[3]
        y = np.empty_like(k)
        for t in range(T):
            kt, vt = k[:, t], v[:, t]
            if wkv == "step_ref":
                ww = pp + u
                p = np.maximum(ww, kt)
                e1, e2 = np.exp(ww - p), np.exp(kt - p)
            else:
                ww = u + kt
                p = np.maximum(pp, ww)
                e1, e2 = np.exp(pp - p), np.exp(ww - p)
            y[:, t] = (e1 * aa + e2 * vt) / (e1 * bb + e2)
            ww2 = pp - decay
            p2 = np.maximum(ww2, kt)
            f1, f2 = np.exp(ww2 - p2), np.exp(kt - p2)
            aa = f1 * aa + f2 * vt
            bb = f1 * bb + f2
            pp = p2
        x = x + _mm(r * y, w[att + "output.weight"])
        state[5 * i + 0] = xx[:, -1].copy()
        state[5 * i + 1], state[5 * i + 2], state[5 * i + 3] = aa, bb, pp

        xx2 = layer_norm(x, w[b + "ln2.weight"], w[b + "ln2.bias"])
        sx2 = _shift(xx2, s[4])
        fk, fr = (w[ffn + n].reshape(-1) for n in ("time_mix_k", "time_mix_r"))
        kx2 = xx2 * fk + sx2 * (1 - fk)
        rx2 = xx2 * fr + sx2 * (1 - fr)
        r2 = _sigmoid(_mm(rx2, w[ffn + "receptance.weight"]))
        kk = np.maximum(_mm(kx2, w[ffn + "key.weight"]), 0) ** 2
        x = x + r2 * _mm(kk, w[ffn + "value.weight"])
        state[5 * i + 4] = xx2[:, -1].copy()
    x = layer_norm(x, w["ln_out.weight"], w["ln_out.bias"])
    return _mm(x, w["head.weight"]), state


def softmax(logits: np.ndarray) -> np.ndarray:
    z = logits.astype(np.float64)
    z = z - z.max(axis=-1, keepdims=True)
    e = np.exp(z)
    return (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)
