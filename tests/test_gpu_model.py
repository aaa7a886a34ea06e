"""RWKV-4 forward on the GPU.

* logits vs the reference's rwkv4_step_ref / forward_batched (golden files)
  within BASELINE's 2e-2 max-abs (fp16 kernels vs fp32 reference);
* packed vs stepped, window composition and batch invariance are
  BIT-identical (reference scripts/test_full_model_packed_vs_stepped.py:77-110,
  test_multi_window_roundtrip.py, test_batched_stepped.py:49-109)."""
import numpy as np
import pytest

from krunch_b200.synth import random_weights

pytestmark = pytest.mark.gpu
LOGIT_TOL = 2e-2


@pytest.fixture(scope="module")
def torch():
    import torch as t
    return t


@pytest.fixture(scope="module")
def tiny(torch):
    from krunch_b200.model import RWKVModel
    return RWKVModel(random_weights(2, 128, 512, 300, seed=0))


def _run(torch, m, tokens, state=None):
    tok = torch.from_numpy(np.ascontiguousarray(tokens, dtype=np.int32)).cuda()
    B, T = tok.shape
    st = m.new_state(B) if state is None else state
    lg = m.new_logits(B, T)
    m.forward_window(tok, st, m.new_workspace(B, T), lg)
    return lg[:, :m.spec.n_vocab].float().view(B, T, -1).cpu().numpy(), st


def test_tiny_logits_vs_reference(torch, tiny, golden_dir):
    g = np.load(golden_dir / "model_tiny.npz")
    st = tiny.new_state(1)
    outs = []
    for t in g["stepped_tokens"]:
        lg, st = _run(torch, tiny, [[t]], st)
        outs.append(lg[0, 0])
    assert np.abs(np.stack(outs) - g["stepped"]).max() <= LOGIT_TOL
    lg, _ = _run(torch, tiny, g["packed_tokens"])
    assert np.abs(lg - g["packed"]).max() <= LOGIT_TOL


def test_169m_logits_vs_reference(torch, golden_dir):
    from krunch_b200.model import RWKVModel
    g = np.load(golden_dir / "model_169m.npz")
    m = RWKVModel(random_weights(12, 768, 3072, 50277, seed=int(g["seed"])))
    st = m.new_state(1)
    outs = []
    for t in g["stepped_tokens"]:
        lg, st = _run(torch, m, [[t]], st)
        outs.append(lg[0, 0])
    o = np.stack(outs)
    assert np.abs(o[:, :256] - g["stepped_head256"]).max() <= LOGIT_TOL
    assert np.abs(o.max(1) - g["stepped_max"]).max() <= LOGIT_TOL
    lg, _ = _run(torch, m, g["packed_tokens"])
    f = lg.reshape(-1, lg.shape[-1])
    assert np.abs(f[:, :256] - g["packed_head256"]).max() <= LOGIT_TOL


def test_169m_full_rows_vs_oracle(torch):
    """Every one of the 50,277 logits of the benchmark model, on 32 stepped
    tokens (B = 1, T = 1 per call) and a packed B = 4 x T = 32 window, against
    the CPU oracle (oracle/rwkv.py: rwkv4_step_ref.py:115-165 and the packed
    forward_batched of batched_rwkv4.py:175-262, pinned to the reference's own
    outputs within 1e-4 by test_oracle_golden): max-abs <= 2e-2 over whole rows."""
    from krunch_b200.model import RWKVModel
    from krunch_b200.synth import zipf_tokens
    from oracle import rwkv
    w = random_weights(12, 768, 3072, 50277, seed=0)
    m = RWKVModel(w)
    stepped = zipf_tokens(32, seed=21)
    st = m.new_state(1)
    outs = []
    for t in stepped:
        lg, st = _run(torch, m, [[t]], st)
        outs.append(lg[0, 0])
    ref, ref_st = rwkv.forward(w, stepped[None])
    d = np.abs(np.stack(outs) - ref[0])
    assert d.shape == (32, 50277) and d.max() <= LOGIT_TOL, d.max()
    # carried state after 32 steps (att_xx / ffn_xx are fp16-rounded on the device)
    got_st = st.cpu().numpy()
    for i in range(12):
        for j in (1, 2):
            a, b = got_st[i, j, 0], ref_st[5 * i + j][0]
            assert np.abs(a - b).max() <= 2e-2 * max(1.0, np.abs(b).max()), (i, j)
    packed = zipf_tokens((4, 32), seed=22)
    lg, _ = _run(torch, m, packed)
    ref, _ = rwkv.forward(w, packed)
    d = np.abs(lg - ref)
    assert d.shape == (4, 32, 50277) and d.max() <= LOGIT_TOL, d.max()
    assert (lg.argmax(-1) == ref.argmax(-1)).mean() >= 0.99


@pytest.mark.parametrize("wkv", ["step_ref", "production"])
def test_packed_equals_stepped_bitwise(torch, wkv):
    from krunch_b200.model import RWKVModel
    m = RWKVModel(random_weights(2, 128, 512, 300, seed=5), wkv=wkv)
    tok = np.random.default_rng(1).integers(0, 300, (3, 20))
    packed, st_p = _run(torch, m, tok)
    st = m.new_state(3)
    steps = []
    for t in range(20):
        lg, st = _run(torch, m, tok[:, t:t + 1], st)
        steps.append(lg[:, 0])
    assert np.array_equal(np.stack(steps, 1), packed)
    assert torch.equal(st, st_p)
    # window composition 7 + 13
    a, st2 = _run(torch, m, tok[:, :7])
    b, st2 = _run(torch, m, tok[:, 7:], st2)
    assert np.array_equal(np.concatenate([a, b], 1), packed)
    # batch invariance: stream 1 alone
    one, _ = _run(torch, m, tok[1:2])
    assert np.array_equal(one[0], packed[1])


def test_production_convention_vs_oracle(torch):
    from krunch_b200.model import RWKVModel
    from oracle import rwkv
    w = random_weights(2, 128, 512, 300, seed=6)
    m = RWKVModel(w, wkv="production")
    tok = np.random.default_rng(2).integers(0, 300, (2, 9))
    lg, _ = _run(torch, m, tok)
    ref, _ = rwkv.forward(w, tok, wkv="production")
    assert np.abs(lg - ref).max() <= LOGIT_TOL


def test_large_window_strips_match_small(torch):
    """Windows of >= 75776 rows run LayerNorm+mix in strips of 4 rows per
    warp; a stream's logits must equal the same stream run alone (1 row per
    warp)."""
    from krunch_b200.model import RWKVModel
    m = RWKVModel(random_weights(2, 128, 512, 300, seed=8))
    tok = np.random.default_rng(3).integers(0, 300, (76, 1000))
    big, st_big = _run(torch, m, tok)
    for b in (0, 37, 75):
        one, st_one = _run(torch, m, tok[b:b + 1])
        assert np.array_equal(one[0], big[b]), b


@pytest.mark.parametrize("wdtype", ["f16", "bf16"])
def test_large_window_odd_streams_with_state(torch, wdtype):
    """Strips of 4 rows are computed two rows at a time; with an odd
    window length a row pair straddles two streams, and the first row of
    every stream takes its token-shift input from the carried state.  The
    result equals the same tokens run as two smaller windows (1 row per
    warp), bit for bit, state included."""
    from krunch_b200.model import RWKVModel
    m = RWKVModel(random_weights(2, 128, 512, 300, seed=10), wdtype=wdtype)
    tok = np.random.default_rng(6).integers(0, 300, (77, 996))
    _, st0 = _run(torch, m, tok[:, :3])
    big, st_big = _run(torch, m, tok[:, 3:], st0.clone())
    assert tok.shape[0] * (tok.shape[1] - 3) >= 148 * 8 * 64
    a, st = _run(torch, m, tok[:, 3:500], st0.clone())
    b, st = _run(torch, m, tok[:, 500:], st)
    assert np.array_equal(np.concatenate([a, b], 1), big)
    assert torch.equal(st, st_big)


@pytest.mark.parametrize("wdtype,B,T", [("f16", 2, 6), ("i8", 2, 6), ("bf16", 2, 6),
                                         ("f16", 3, 19), ("bf16", 3, 19)])
def test_wide_rows_vs_oracle_and_stepped(torch, wdtype, B, T):
    """C = 2048 (the 1.5B width) runs LayerNorm+mix in the streaming kernel
    (fp16, bf16 and w8a8 outputs; ragged B x T): logits near the oracle,
    packed == stepped bit for bit."""
    from krunch_b200.model import RWKVModel
    from oracle import rwkv
    w = random_weights(2, 2048, 8192, 300, seed=9)
    m = RWKVModel(w, wdtype=wdtype)
    tok = np.random.default_rng(5).integers(0, 300, (B, T))
    packed, st_p = _run(torch, m, tok)
    ref, _ = rwkv.forward(w, tok, wdtype=wdtype if wdtype != "f16" else "f32")
    d = np.abs(packed - ref)
    if wdtype == "bf16":
        assert d.max() <= 5e-2
    elif wdtype == "f16":
        assert d.max() <= LOGIT_TOL
    else:
        assert d.mean() <= 2e-2 and d.max() <= 0.15
    st = m.new_state(B)
    steps = []
    for t in range(T):
        lg, st = _run(torch, m, tok[:, t:t + 1], st)
        steps.append(lg[:, 0])
    assert np.array_equal(np.stack(steps, 1), packed)
    assert torch.equal(st, st_p)
