"""Generate peaked_169m_tokens.npy: token streams sampled from a peaked model.

The size-parity tests need a model whose predictions carry information: on
random-init RWKV-4-169M weights the head logits have a standard deviation of
about 0.55, every 16-bit count except the argmax's is 1 and any model —
including a broken one — codes a stream at ~16 bits per token.  Scaling the
seeded head by HEAD_SCALE (= 8) gives logits of standard deviation ~4.4, and
sampling each stream from that model itself (seeded, temperature 1) makes
the model the stream's true generator: its code length is then the stream's
entropy (~5-7 bits per token), and any deviation of the logits (a zeroed
layer, a wrong state carry) costs a measurable KL excess.

Sampling runs the CPU oracle (oracle/rwkv.py, itself pinned to the
reference's rwkv4_step_ref within 1e-4) one token at a time from the BOS
token 0 for B streams in lockstep; it is run by hand:
    python tests/golden/make_peaked.py
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from krunch_b200.synth import RWKV4_169M, random_weights  # noqa: E402
from oracle import rwkv  # noqa: E402

HEAD_SCALE = 8.0
WEIGHT_SEED = 0
SAMPLE_SEED = 7
B, T = 4, 512


def peaked_weights() -> dict:
    w = random_weights(**RWKV4_169M, seed=WEIGHT_SEED)
    w["head.weight"] = w["head.weight"] * np.float32(HEAD_SCALE)
    return w


def main() -> None:
    w = peaked_weights()
    rng = np.random.default_rng(SAMPLE_SEED)
    st = rwkv.init_state(w, B)
    cur = np.zeros((B, 1), np.int64)
    toks = np.zeros((B, T), np.int32)
    V = w["emb.weight"].shape[0]
    for t in range(T):
        lg, st = rwkv.forward(w, cur, st)
        p = rwkv.softmax(lg[:, 0]).astype(np.float64)
        p /= p.sum(axis=1, keepdims=True)
        for b in range(B):
            toks[b, t] = rng.choice(V, p=p[b])
        cur = toks[:, t:t + 1].astype(np.int64)
    np.save(HERE / "peaked_169m_tokens.npy", toks)
    print("wrote", toks.shape)


if __name__ == "__main__":
    main()
