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


# ---- w8a8 (the build's KB_I8 model; the reference has no w8a8 path) --------

def quantize_weight(W: np.ndarray):
    """[in, out] matrix -> int8 [out, in] and fp16 factor per output channel:
    s = fp16(max|w| / 127), q = clamp(rint(w / s), -127, 127), from the fp16
    weights the device holds."""
    w16 = np.asarray(W, np.float32).T.astype(np.float16).astype(np.float32)
    amax = np.abs(w16).max(axis=1)
    s = (amax / np.float32(127)).astype(np.float32).astype(np.float16)
    sf = s.astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(sf[:, None] > 0, np.rint(w16 / sf[:, None]), 0)
    return np.clip(q, -127, 127).astype(np.int8), s


def quantize_rows(x: np.ndarray):
    """fp32 rows [R, K] -> int8 [R, K] and fp32 factor per row, from the fp16
    rounding of x: q = clamp(rint(a * (127 / amax)), -127, 127), factor amax / 127."""
    a = np.asarray(x, np.float32).astype(np.float16).astype(np.float32)
    amax = np.abs(a).max(axis=1)
    inv = np.where(amax > 0, np.float32(127) / np.where(amax > 0, amax, 1), 0).astype(np.float32)
    q = np.clip(np.rint(a * inv[:, None]), -127, 127).astype(np.int8)
    return q, (amax / np.float32(127)).astype(np.float32)


def bf16_round(a: np.ndarray) -> np.ndarray:
    """float32 -> nearest bf16 (ties to even), returned as float32."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def _mm8(x: np.ndarray, Wq) -> np.ndarray:
    """w8a8 product: exact integer accumulation, then (acc * sa) * sw."""
    q, s = Wq
    B, T, C = x.shape
    qa, sa = quantize_rows(x.reshape(B * T, C))
    acc = qa.astype(np.int64) @ q.astype(np.int64).T
    y = (acc.astype(np.float32) * sa[:, None]) * s.astype(np.float32)[None, :]
    return y.reshape(B, T, q.shape[0])


def forward(w: dict, tokens: np.ndarray, state: list[np.ndarray] | None = None,
            wkv: str = "step_ref", wdtype: str = "f32") -> tuple[np.ndarray, list[np.ndarray]]:
    """tokens int [B, T] -> (logits fp32 [B, T, V], new state).

    wdtype "bf16" rounds every matrix and every GEMM input to bf16 (the
    device's KB_BF16 model); wdtype "i8" runs the w8a8 model: every matrix
    product through _mm8; in both,
    the activations the device keeps in fp16 (embedding, residual stream,
    LayerNorm outputs, sigmoid gates) rounded to fp16 where the device rounds
    them, so that the per-row quantisation sees the device's values."""
    h = ((lambda a: a.astype(np.float16).astype(np.float32)) if wdtype in ("i8", "bf16")
         else (lambda a: a))
    if wdtype == "bf16":
        bcache = {}

        def mm(x, name):
            if name not in bcache:
                bcache[name] = bf16_round(w[name])
            return _mm(bf16_round(x), bcache[name])
    elif wdtype == "i8":
        qcache = {}

        def mm(x, name):
            if name not in qcache:
                qcache[name] = quantize_weight(w[name])
            return _mm8(x, qcache[name])
    else:
        def mm(x, name):
            return _mm(x, w[name])
    tok = np.asarray(tokens)
    if tok.ndim == 1:
        tok = tok[None]
    B, T = tok.shape
    if state is None:
        state = init_state(w, B)
    state = [s.copy() for s in state]
    x = h(w["emb.weight"][tok].astype(np.float32))
    for i in range(n_layer_of(w)):
        b, att, ffn = f"blocks.{i}.", f"blocks.{i}.att.", f"blocks.{i}.ffn."
        s = state[5 * i:5 * i + 5]
        xx = h(layer_norm(x, w[b + "ln1.weight"], w[b + "ln1.bias"]))
        sx = _shift(xx, s[0])
        mk, mv, mr = (w[att + n].reshape(-1) for n in ("time_mix_k", "time_mix_v", "time_mix_r"))
        kx = xx * mk + sx * (1 - mk)
        vx = xx * mv + sx * (1 - mv)
        rx = xx * mr + sx * (1 - mr)
        r = h(_sigmoid(mm(rx, att + "receptance.weight")))
        k = mm(kx, att + "key.weight")
        v = mm(vx, att + "value.weight")
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
        x = h(x + mm(r * y, att + "output.weight"))
        state[5 * i + 0] = xx[:, -1].copy()
        state[5 * i + 1], state[5 * i + 2], state[5 * i + 3] = aa, bb, pp

        xx2 = h(layer_norm(x, w[b + "ln2.weight"], w[b + "ln2.bias"]))
        sx2 = _shift(xx2, s[4])
        fk, fr = (w[ffn + n].reshape(-1) for n in ("time_mix_k", "time_mix_r"))
        kx2 = xx2 * fk + sx2 * (1 - fk)
        rx2 = xx2 * fr + sx2 * (1 - fr)
        r2 = h(_sigmoid(mm(rx2, ffn + "receptance.weight")))
        kk = np.maximum(mm(kx2, ffn + "key.weight"), 0) ** 2
        x = h(x + r2 * mm(kk, ffn + "value.weight"))
        state[5 * i + 4] = xx2[:, -1].copy()
    x = h(layer_norm(x, w["ln_out.weight"], w["ln_out.bias"]))
    return mm(x, "head.weight"), state


def softmax(logits: np.ndarray) -> np.ndarray:
    z = logits.astype(np.float64)
    z = z - z.max(axis=-1, keepdims=True)
    e = np.exp(z)
    return (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)
