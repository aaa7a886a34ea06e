"""Generate the golden fixtures in this directory from the reference's own code.

Runs the UNMODIFIED reference Python (krunch_ac/cpu_reference.py,
krunch_ac/cdf.py, scripts/rwkv4_step_ref.py, krunch/batched_rwkv4.py with
KRUNCH_PURE_WKV=1) on seeded inputs and stores what it produced:

* coder_cases.json — for every shape/seed of the reference's own coder tests
  (tests/test_ac_reference.py:63-139, tests/test_ac_kernel_gpu.py:57-66) at
  CDF totals 2^24 (the reference's) and 2^16: the sha256 of the reference CDF
  and the bitstream cpu_reference.encode wrote for it.
* cdf_cases.json — sha256 of probs_to_cdf outputs, plus two small CDFs in full.
* model_tiny.npz / model_169m.npz — step_ref logits (stepped, B=1) and
  forward_batched logits (packed, B=2) on seeded random-init weights
  (krunch_b200.synth.random_weights) — full rows for the tiny model, the first
  256 logits and row summaries for RWKV-4-169M.

Needs the reference tree (the directory in $KRUNCH_REFERENCE) and
torch; it is run by hand, not by the test suite:
    KRUNCH_REFERENCE=<reference checkout> python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

from krunch_b200.synth import random_weights  # noqa: E402

REF = Path(os.environ.get("KRUNCH_REFERENCE", "reference"))

# (N, V, seed) of tests/test_ac_reference.py:63-69 and test_ac_kernel_gpu.py:57-63
CODER_SHAPES = [(1, 4, 10), (16, 64, 11), (256, 256, 12), (1024, 1024, 13), (4096, 50277, 14),
                (1, 4, 0), (8, 32, 1), (256, 256, 2), (1024, 1024, 3), (256, 50277, 4)]
TINY = dict(n_layer=2, n_embd=128, n_ffn=512, n_vocab=300)


def rand_probs(N, V, seed):
    """tests/test_ac_reference.py:14-18"""
    rng = np.random.default_rng(seed)
    p = rng.random((N, V)).astype(np.float32)
    p /= p.sum(axis=1, keepdims=True)
    return p


def sample_symbols(p, seed):
    """tests/test_ac_reference.py:71-76"""
    rng = np.random.default_rng(seed + 100)
    cum = np.cumsum(p, axis=1)
    u = rng.random((p.shape[0], 1)).astype(np.float32)
    return (u < cum).argmax(axis=1).astype(np.int32)


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def ref_cdf(cdf_mod, p, bits):
    cdf_mod.T = 1 << bits  # probs_to_cdf reads the module global (cdf.py:19,50,60)
    try:
        return cdf_mod.probs_to_cdf(p)
    finally:
        cdf_mod.T = 1 << 24


def coder_and_cdf():
    from krunch_ac import cdf as cdf_mod
    from krunch_ac import cpu_reference as rc

    coder, cdfs = [], []
    for bits in (24, 16):
        for N, V, seed in CODER_SHAPES:
            p = rand_probs(N, V, seed)
            sym = sample_symbols(p, seed)
            c = ref_cdf(cdf_mod, p, bits)
            bs = rc.encode(c, sym)
            assert (rc.decode(bs, c) == sym).all()
            coder.append(dict(N=N, V=V, seed=seed, bits=bits, cdf_sha256=sha(c),
                              bitstream=bs.hex()))
            print(f"coder bits={bits} N={N} V={V} -> {len(bs)} B", flush=True)
        # edge cases of tests/test_ac_reference.py:79-139
        p = rand_probs(100, 50, 20)
        sym = np.zeros(100, np.int32)
        c = ref_cdf(cdf_mod, p, bits)
        coder.append(dict(name="all_same_symbol", bits=bits, cdf_sha256=sha(c),
                          bitstream=rc.encode(c, sym).hex()))
        V, N = 200, 50
        p = np.full((N, V), 1e-6, np.float32)
        p[:, 0] = 1.0 - 1e-6 * (V - 1)
        p /= p.sum(axis=1, keepdims=True)
        c = ref_cdf(cdf_mod, p, bits)
        coder.append(dict(name="low_prob_symbol", bits=bits, cdf_sha256=sha(c),
                          bitstream=rc.encode(c, np.full(N, 199, np.int32)).hex()))
        N, V = 2048, 1024
        p = np.full((N, V), 1.0, np.float32)
        p[:, 0] = 1000.0
        p /= p.sum(axis=1, keepdims=True)
        c = ref_cdf(cdf_mod, p, bits)
        coder.append(dict(name="peaky", bits=bits, cdf_sha256=sha(c),
                          bitstream=rc.encode(c, np.zeros(N, np.int32)).hex()))
        p = np.full((1, 100), 1e-9, np.float32)
        p[0, 50] = 1.0
        p /= p.sum()
        cdfs.append(dict(name="extreme", bits=bits, cdf=ref_cdf(cdf_mod, p, bits)[0].tolist()))
        p = rand_probs(3, 40, 5)
        cdfs.append(dict(name="small_random", bits=bits, cdf=ref_cdf(cdf_mod, p, bits).tolist()))
        for N, V, seed in [(64, 256, 1), (16, 50277, 7)]:
            c = ref_cdf(cdf_mod, rand_probs(N, V, seed), bits)
            cdfs.append(dict(N=N, V=V, seed=seed, bits=bits, cdf_sha256=sha(c)))
    (HERE / "coder_cases.json").write_text(json.dumps(coder, indent=0))
    (HERE / "cdf_cases.json").write_text(json.dumps(cdfs, indent=0))


def _shim(w_np, n_layer, n_embd):
    import torch
    w = {k: torch.from_numpy(v.copy()) for k, v in w_np.items()}
    dd = types.SimpleNamespace(atype=torch.float32, device="cpu")
    args = types.SimpleNamespace(n_layer=n_layer, n_embd=n_embd, n_att=n_embd)
    return types.SimpleNamespace(w=w, args=args, strategy=[dd] * n_layer, version=4)


def model_logits(cfg, stepped_tokens, packed_tokens, full: bool, out: Path, seed: int = 0):
    import torch
    torch.set_num_threads(os.cpu_count() or 1)
    os.environ["KRUNCH_PURE_WKV"] = "1"
    sys.path.insert(0, str(REF / "scripts"))
    import rwkv4_step_ref as sr
    from krunch import batched_rwkv4 as bw

    w = random_weights(**cfg, seed=seed)
    m = _shim(w, cfg["n_layer"], cfg["n_embd"])
    with torch.no_grad():
        st = sr.init_state_step(m, device="cpu")
        step = []
        for tok in stepped_tokens:
            lg, st = sr.step_one(m, int(tok), st)
            step.append(lg.float().numpy())
        step = np.stack(step)
        toks = torch.as_tensor(packed_tokens, dtype=torch.long)
        state = bw.init_state_batched(m, toks.shape[0], device="cpu")
        packed, _ = bw.forward_batched(m, toks, state, full_output=True)
        packed = packed.float().numpy()
    rec = dict(stepped_tokens=np.asarray(stepped_tokens, np.int32),
               packed_tokens=np.asarray(packed_tokens, np.int32), seed=np.int64(seed))
    for name, arr in (("stepped", step), ("packed", packed)):
        flat = arr.reshape(-1, arr.shape[-1])
        if full:
            rec[name] = arr.astype(np.float32)
        else:
            rec[name + "_head256"] = flat[:, :256].astype(np.float32)
            rec[name + "_max"] = flat.max(axis=1)
            rec[name + "_argmax"] = flat.argmax(axis=1).astype(np.int32)
            z = flat.astype(np.float64)
            rec[name + "_lse"] = (np.log(np.exp(z - z.max(1, keepdims=True)).sum(1))
                                  + z.max(1)).astype(np.float64)
    np.savez_compressed(out, **rec)
    print(f"wrote {out.name}", flush=True)


def main():
    sys.path.insert(0, str(REF))
    coder_and_cdf()
    rng = np.random.default_rng(123)
    model_logits(TINY, rng.integers(0, TINY["n_vocab"], 12), rng.integers(0, TINY["n_vocab"], (2, 12)),
                 True, HERE / "model_tiny.npz")
    big = dict(n_layer=12, n_embd=768, n_ffn=3072, n_vocab=50277)
    model_logits(big, [0, 100, 1000, 5, 42, 9999], rng.integers(0, 50277, (2, 6)), False,
                 HERE / "model_169m.npz")


if __name__ == "__main__":
    main()
