"""The CPU oracle against fixtures the reference's own code produced.

Golden files (tests/golden/, made by tests/golden/make_golden.py from
krunch_ac/cpu_reference.py, krunch_ac/cdf.py, scripts/rwkv4_step_ref.py and
krunch/batched_rwkv4.py) pin:
  * oracle.cdf_spec.probs_to_cdf == reference probs_to_cdf   (sha256, 2^16 and 2^24)
  * oracle.coder.encode          == reference encode bytes   (same CDF)
  * oracle.coder.decode round trip
  * oracle.rwkv logits           == step_ref / forward_batched logits (<= 1e-4)
"""
import json

import numpy as np
import pytest

from helpers import named_case, rand_probs, sample_symbols, sha
from oracle import cdf_spec, coder, rwkv
from krunch_b200.synth import random_weights

CPU_MAX_ELEMS = 16_000_000  # keep the CPU suite to minutes


def _cases(golden_dir, name):
    return json.loads((golden_dir / name).read_text())


def _coder_params(golden_dir):
    out = []
    for c in _cases(golden_dir, "coder_cases.json"):
        if "name" in c:
            out.append(pytest.param(c, id=f"{c['name']}-b{c['bits']}"))
        elif c["N"] * c["V"] <= CPU_MAX_ELEMS:
            out.append(pytest.param(c, id=f"N{c['N']}-V{c['V']}-s{c['seed']}-b{c['bits']}"))
    return out


def pytest_generate_tests(metafunc):
    if "coder_case" in metafunc.fixturenames:
        from conftest import GOLDEN
        metafunc.parametrize("coder_case", _coder_params(GOLDEN))


def _probs_syms(case):
    if "name" in case:
        return named_case(case["name"])
    p = rand_probs(case["N"], case["V"], case["seed"])
    return p, sample_symbols(p, case["seed"])


def test_coder_matches_reference_bytes(coder_case):
    p, sym = _probs_syms(coder_case)
    cdf = cdf_spec.probs_to_cdf(p, coder_case["bits"])
    assert sha(cdf) == coder_case["cdf_sha256"], "numpy CDF restatement differs from reference"
    bs = coder.encode(cdf, sym)
    assert bs.hex() == coder_case["bitstream"], "oracle coder bytes differ from reference"
    assert (coder.decode(bs, cdf) == sym).all()


def test_stateful_decoder_matches_one_shot(golden_dir):
    p = rand_probs(64, 300, 3)
    sym = sample_symbols(p, 3)
    cdf = cdf_spec.probs_to_cdf(p, 16)
    bs = coder.encode(cdf, sym)
    dec = coder.RangeDecoder(bs)
    assert [dec.decode_symbol(cdf[i]) for i in range(64)] == sym.tolist()


def test_cdf_hashes_and_full_rows(golden_dir):
    for c in _cases(golden_dir, "cdf_cases.json"):
        if "cdf" in c:
            if c["name"] == "extreme":
                p = np.full((1, 100), 1e-9, np.float32)
                p[0, 50] = 1.0
                p /= p.sum()
            else:
                p = rand_probs(3, 40, 5)
            got = cdf_spec.probs_to_cdf(p, c["bits"])
            assert got.reshape(-1).tolist() == np.asarray(c["cdf"]).reshape(-1).tolist()
        else:
            got = cdf_spec.probs_to_cdf(rand_probs(c["N"], c["V"], c["seed"]), c["bits"])
            assert sha(got) == c["cdf_sha256"]


@pytest.mark.parametrize("bits", [16, 24])
def test_fixed_order_cdf_invariants_and_closeness(bits):
    """The kernel-order CDF (C oracle) obeys cdf.py's invariants and differs
    from numpy's pairwise-summed spec only through last-bit sum rounding."""
    p = rand_probs(64, 256, 1)
    a = coder.cdf_from_probs(p, bits).astype(np.int64)
    b = cdf_spec.probs_to_cdf(p, bits).astype(np.int64)
    assert (a[:, 0] == 0).all() and (a[:, -1] == 1 << bits).all()
    assert (np.diff(a, axis=1) >= 1).all()
    ca, cb = np.diff(a, axis=1), np.diff(b, axis=1)
    am = p.argmax(axis=1)
    mask = np.ones_like(ca, bool)
    mask[np.arange(len(am)), am] = False
    assert np.abs(ca - cb)[mask].max() <= 1


def test_cdf_from_logits_invariants():
    rng = np.random.default_rng(0)
    for V, bits in [(4, 16), (300, 16), (50277, 24), (50277, 16)]:
        x = (rng.standard_normal((3, V)) * 3).astype(np.float16)
        c = coder.cdf_from_logits(x, bits).astype(np.int64)
        assert (c[:, 0] == 0).all() and (c[:, -1] == 1 << bits).all()
        assert (np.diff(c, axis=1) >= 1).all()
        # the most probable symbol has the widest bin
        w = np.diff(c, axis=1)
        assert (w.argmax(axis=1) == x.astype(np.float32).argmax(axis=1)).all()


def test_lohi_matches_full_cdf():
    x = (np.random.default_rng(1).standard_normal((7, 1000)) * 2).astype(np.float16)
    s = np.random.default_rng(2).integers(0, 1000, 7).astype(np.int32)
    c = coder.cdf_from_logits(x, 16)
    lh = coder.lohi_from_logits(x, s, 16)
    assert (lh[:, 0] == c[np.arange(7), s]).all() and (lh[:, 1] == c[np.arange(7), s + 1]).all()
    bs1 = coder.encode(c.astype(np.uint32), s)
    assert coder.encode_lohi(lh, 16) == bs1


def test_expf_accuracy():
    x = np.linspace(-86, 0, 20001).astype(np.float32)
    e = coder.expf(x)
    ref = np.exp(x.astype(np.float64))
    assert np.max(np.abs(e - ref) / ref) < 7e-6
    assert coder.expf([-87.0, -np.inf])[0] == 0.0


def test_rwkv_oracle_tiny_matches_reference(golden_dir):
    g = np.load(golden_dir / "model_tiny.npz")
    w = random_weights(2, 128, 512, 300, seed=int(g["seed"]))
    st = rwkv.init_state(w, 1)
    outs = []
    for t in g["stepped_tokens"]:
        lg, st = rwkv.forward(w, np.array([[t]]), st)
        outs.append(lg[0, 0])
    assert np.abs(np.stack(outs) - g["stepped"]).max() < 1e-4
    lg, _ = rwkv.forward(w, g["packed_tokens"])
    assert np.abs(lg - g["packed"]).max() < 1e-4


def test_rwkv_oracle_window_composition():
    w = random_weights(2, 128, 512, 300, seed=3)
    tok = np.random.default_rng(0).integers(0, 300, (2, 10))
    full, _ = rwkv.forward(w, tok)
    a, st = rwkv.forward(w, tok[:, :4])
    b, _ = rwkv.forward(w, tok[:, 4:], st)
    assert np.abs(np.concatenate([a, b], 1) - full).max() < 1e-5


@pytest.mark.slow
def test_rwkv_oracle_169m_matches_reference(golden_dir):
    g = np.load(golden_dir / "model_169m.npz")
    w = random_weights(12, 768, 3072, 50277, seed=int(g["seed"]))
    st = rwkv.init_state(w, 1)
    outs = []
    for t in g["stepped_tokens"]:
        lg, st = rwkv.forward(w, np.array([[t]]), st)
        outs.append(lg[0, 0])
    o = np.stack(outs)
    assert np.abs(o[:, :256] - g["stepped_head256"]).max() < 1e-4
    assert (o.argmax(1) == g["stepped_argmax"]).all()
    lg, _ = rwkv.forward(w, g["packed_tokens"])
    f = lg.reshape(-1, lg.shape[-1])
    assert np.abs(f[:, :256] - g["packed_head256"]).max() < 1e-4
