"""Seeded synthetic weights and inputs for the benchmark configurations.

No pretrained RWKV-4 weights, tokenizer file or corpus ship with this build,
so every measurement runs on the seeded stand-ins below (numpy PCG64):

* ``random_weights`` — RWKV-4 random init in the reference's ``model.w``
  layout (matrices ``[in, out]``, mixes ``[C]``): N(0, 0.02) for every matrix
  including emb and head, time_decay U[-5, 0], time_first U[-1, 1], time-mix
  vectors U[0, 1), LayerNorm gamma 1 / beta 0.  Tensors are drawn in a fixed
  order (emb; per layer: time_decay, time_first, att mixes k/v/r, key, value,
  receptance, output, ffn mixes k/r, key, value, receptance; head).
* ``zipf_tokens`` — i.i.d. Zipf(s) ranks over the vocabulary mapped through a
  seeded permutation (the compress / decompress token workloads).
* ``markov_text`` — order-2 character Markov text over printable ASCII plus
  newline, transition rows Dirichlet(0.1) (the CPU plumbing workload).
* ``log_lines`` — ``"{ISO-8601} {IPv4} {LEVEL} {words}\\n"`` lines over a
  2,000-word Zipf(1.2) vocabulary (the box-level workload).
"""
from __future__ import annotations

import datetime as _dt

import numpy as np

RWKV4_169M = dict(n_layer=12, n_embd=768, n_ffn=3072, n_vocab=50277)
RWKV4_1B5 = dict(n_layer=24, n_embd=2048, n_ffn=8192, n_vocab=50277)


def random_weights(n_layer: int, n_embd: int, n_ffn: int, n_vocab: int, seed: int = 0,
                   std: float = 0.02) -> dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    C, F, V = n_embd, n_ffn, n_vocab

    def normal(*shape):
        a = rng.standard_normal(shape, dtype=np.float32)
        a *= np.float32(std)
        return a

    def unif(lo, hi, n):
        return (rng.random(n, dtype=np.float32) * np.float32(hi - lo) + np.float32(lo)).astype(
            np.float32)

    w: dict[str, np.ndarray] = {}
    w["emb.weight"] = normal(V, C)
    ones, zeros = np.ones(C, np.float32), np.zeros(C, np.float32)
    for i in range(n_layer):
        b, att, ffn = f"blocks.{i}.", f"blocks.{i}.att.", f"blocks.{i}.ffn."
        w[b + "ln1.weight"], w[b + "ln1.bias"] = ones.copy(), zeros.copy()
        w[b + "ln2.weight"], w[b + "ln2.bias"] = ones.copy(), zeros.copy()
        w[att + "time_decay"] = unif(-5.0, 0.0, C)
        w[att + "time_first"] = unif(-1.0, 1.0, C)
        w[att + "time_mix_k"] = unif(0.0, 1.0, C)
        w[att + "time_mix_v"] = unif(0.0, 1.0, C)
        w[att + "time_mix_r"] = unif(0.0, 1.0, C)
        w[att + "key.weight"] = normal(C, C)
        w[att + "value.weight"] = normal(C, C)
        w[att + "receptance.weight"] = normal(C, C)
        w[att + "output.weight"] = normal(C, C)
        w[ffn + "time_mix_k"] = unif(0.0, 1.0, C)
        w[ffn + "time_mix_r"] = unif(0.0, 1.0, C)
        w[ffn + "key.weight"] = normal(C, F)
        w[ffn + "value.weight"] = normal(F, C)
        w[ffn + "receptance.weight"] = normal(C, C)
    w["ln_out.weight"], w["ln_out.bias"] = ones.copy(), zeros.copy()
    w["head.weight"] = normal(C, V)
    return w


def random_weights_device(n_layer: int, n_embd: int, n_ffn: int, n_vocab: int, seed: int = 0,
                          std: float = 0.02, device="cuda") -> dict[str, np.ndarray]:
    """The distribution of ``random_weights`` drawn by torch's generator on a
    CUDA device (seconds instead of minutes for the 1.5B shapes), returned
    as numpy float32 arrays in the same layout.  A different stream of
    numbers than ``random_weights`` for the same seed."""
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    C, F, V = n_embd, n_ffn, n_vocab

    def normal(*shape):
        return (torch.randn(shape, generator=g, device=device) * std).cpu().numpy()

    def unif(lo, hi, n):
        return (torch.rand(n, generator=g, device=device) * (hi - lo) + lo).cpu().numpy()

    w: dict[str, np.ndarray] = {"emb.weight": normal(V, C)}
    ones, zeros = np.ones(C, np.float32), np.zeros(C, np.float32)
    for i in range(n_layer):
        b, att, ffn = f"blocks.{i}.", f"blocks.{i}.att.", f"blocks.{i}.ffn."
        w[b + "ln1.weight"], w[b + "ln1.bias"] = ones.copy(), zeros.copy()
        w[b + "ln2.weight"], w[b + "ln2.bias"] = ones.copy(), zeros.copy()
        w[att + "time_decay"] = unif(-5.0, 0.0, C)
        w[att + "time_first"] = unif(-1.0, 1.0, C)
        for n in ("time_mix_k", "time_mix_v", "time_mix_r"):
            w[att + n] = unif(0.0, 1.0, C)
        for n in ("key", "value", "receptance", "output"):
            w[att + n + ".weight"] = normal(C, C)
        w[ffn + "time_mix_k"] = unif(0.0, 1.0, C)
        w[ffn + "time_mix_r"] = unif(0.0, 1.0, C)
        w[ffn + "key.weight"] = normal(C, F)
        w[ffn + "value.weight"] = normal(F, C)
        w[ffn + "receptance.weight"] = normal(C, C)
    w["ln_out.weight"], w["ln_out.bias"] = ones.copy(), zeros.copy()
    w["head.weight"] = normal(C, V)
    return w


def zipf_tokens(shape, vocab: int = 50277, s: float = 1.1, seed: int = 0) -> np.ndarray:
    rng = np.random.default_rng(seed)
    ranks = np.arange(1, vocab + 1, dtype=np.float64)
    p = ranks ** (-s)
    p /= p.sum()
    perm = rng.permutation(vocab)
    r = rng.choice(vocab, size=shape, p=p)
    return perm[r].astype(np.int32)


def markov_text(n_bytes: int, seed: int = 1, alpha: float = 0.1) -> bytes:
    alphabet = np.array([*range(0x20, 0x7F), 0x0A], dtype=np.uint8)  # 96 symbols
    k = len(alphabet)
    rng = np.random.default_rng(seed)
    table = rng.dirichlet(np.full(k, alpha), size=k * k).astype(np.float64)
    cum = np.cumsum(table, axis=1)
    u = rng.random(n_bytes)
    out = np.empty(n_bytes, dtype=np.uint8)
    a, b = 0, 0
    for i in range(n_bytes):
        row = cum[a * k + b]
        c = int(np.searchsorted(row, u[i] * row[-1], side="right"))
        c = min(c, k - 1)
        out[i] = alphabet[c]
        a, b = b, c
    return out.tobytes()


def _words(rng, n: int) -> list[str]:
    letters = np.frombuffer(b"abcdefghijklmnopqrstuvwxyz", dtype=np.uint8)
    lens = rng.integers(2, 11, size=n)
    return [letters[rng.integers(0, 26, size=L)].tobytes().decode() for L in lens]


def log_lines(n_bytes: int, seed: int = 4, vocab_words: int = 2000, s: float = 1.2) -> bytes:
    rng = np.random.default_rng(seed)
    words = _words(rng, vocab_words)
    p = np.arange(1, vocab_words + 1, dtype=np.float64) ** (-s)
    p /= p.sum()
    levels = ["INFO", "WARN", "ERROR", "DEBUG"]
    lp = np.array([0.7, 0.15, 0.05, 0.10])
    t0 = _dt.datetime(2026, 1, 1, tzinfo=_dt.timezone.utc)
    parts: list[bytes] = []
    total = 0
    sec = 0
    while total < n_bytes:
        n = 4096
        dts = rng.integers(0, 3, size=n).cumsum() + sec
        sec = int(dts[-1])
        ips = rng.integers(1, 255, size=(n, 4))
        lv = rng.choice(4, size=n, p=lp)
        nw = rng.integers(3, 13, size=n)
        wi = rng.choice(vocab_words, size=int(nw.sum()), p=p)
        pos = 0
        lines = []
        for j in range(n):
            ts = (t0 + _dt.timedelta(seconds=int(dts[j]))).strftime("%Y-%m-%dT%H:%M:%SZ")
            msg = " ".join(words[x] for x in wi[pos:pos + nw[j]])
            pos += nw[j]
            a, b, c, d = ips[j]
            lines.append(f"{ts} {a}.{b}.{c}.{d} {levels[lv[j]]} {msg}\n")
        blob = "".join(lines).encode()
        parts.append(blob)
        total += len(blob)
    return b"".join(parts)[:n_bytes]
