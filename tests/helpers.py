"""Shared seeded generators for the tests (the reference's own test recipes)."""
import hashlib

import numpy as np


def rand_probs(N, V, seed):
    """tests/test_ac_reference.py:14-18 of the reference."""
    rng = np.random.default_rng(seed)
    p = rng.random((N, V)).astype(np.float32)
    p /= p.sum(axis=1, keepdims=True)
    return p


def sample_symbols(p, seed):
    """tests/test_ac_reference.py:71-76 of the reference."""
    rng = np.random.default_rng(seed + 100)
    cum = np.cumsum(p, axis=1)
    u = rng.random((p.shape[0], 1)).astype(np.float32)
    return (u < cum).argmax(axis=1).astype(np.int32)


def named_case(name):
    """Edge cases of tests/test_ac_reference.py:79-139 -> (probs, symbols)."""
    if name == "all_same_symbol":
        return rand_probs(100, 50, 20), np.zeros(100, np.int32)
    if name == "low_prob_symbol":
        V, N = 200, 50
        p = np.full((N, V), 1e-6, np.float32)
        p[:, 0] = 1.0 - 1e-6 * (V - 1)
        p /= p.sum(axis=1, keepdims=True)
        return p, np.full(N, 199, np.int32)
    if name == "peaky":
        N, V = 2048, 1024
        p = np.full((N, V), 1.0, np.float32)
        p[:, 0] = 1000.0
        p /= p.sum(axis=1, keepdims=True)
        return p, np.zeros(N, np.int32)
    raise KeyError(name)


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def random_logits(rows, V, seed, scale=2.0, dtype=np.float16):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((rows, V)) * scale).astype(dtype)
