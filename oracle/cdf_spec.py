"""numpy restatement of krunch_ac/cdf.py:probs_to_cdf — TEST INFRASTRUCTURE ONLY.

Same numpy operations in the same order as the reference (cdf.py:52-74), so
it reproduces the reference's CDF bit for bit on the same numpy build; the
total T = 2^bits is a parameter (the reference reads a module global, 2^24).
"""
from __future__ import annotations

import numpy as np


def probs_to_cdf(probs: np.ndarray, bits: int = 24) -> np.ndarray:
    T = 1 << bits
    if probs.ndim == 1:
        probs = probs.reshape(1, -1)
    N, V = probs.shape
    assert V < T
    p = probs.astype(np.float32, copy=False)
    p = p / np.maximum(p.sum(axis=1, keepdims=True), np.float32(1e-30))
    counts = np.floor(p * (T - V)).astype(np.int64) + 1
    deficit = T - counts.sum(axis=1)
    if int(deficit.max()) > 0 or int(deficit.min()) < 0:
        counts[np.arange(N), p.argmax(axis=1)] += deficit
    assert (counts.sum(axis=1) == T).all() and (counts > 0).all()
    cdf = np.zeros((N, V + 1), dtype=np.uint32)
    cdf[:, 1:] = np.cumsum(counts, axis=1).astype(np.uint32)
    return cdf
