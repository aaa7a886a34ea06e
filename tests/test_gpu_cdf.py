"""Fused logits -> integer CDF kernel: bit-exact against the C oracle (same
fixed reduction order), batch-invariant (scripts/test_det_softmax_cdf.py:18-41
of the reference), and the fused decode step round-trips."""
import numpy as np
import pytest

from helpers import random_logits
from oracle import coder

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as t
    return t


def _cdf_gpu(torch, logits_np, bits, mode=1, stride=None, symbols=None):
    from krunch_b200 import _native as N
    rows, V = logits_np.shape
    stride = stride or V
    buf = np.zeros((rows, stride), np.float16)
    buf[:, :V] = logits_np
    x = torch.from_numpy(buf).cuda()
    if mode == N.KB_CDF_LOHI:
        out = torch.empty((rows, 2), dtype=torch.int32, device="cuda")
        sym = torch.from_numpy(symbols.astype(np.int32)).cuda()
        N.call("kb_cdf_rows", x.data_ptr(), stride, rows, V, bits, mode, None, 0, sym.data_ptr(),
               out.data_ptr(), N.stream_ptr())
        return out.cpu().numpy().view(np.uint32)
    out = torch.empty((rows, V + 1), dtype=torch.int32, device="cuda")
    N.call("kb_cdf_rows", x.data_ptr(), stride, rows, V, bits, mode, None, 0, None, out.data_ptr(),
           N.stream_ptr())
    return out.cpu().numpy()


@pytest.mark.parametrize("bits", [16, 24])
@pytest.mark.parametrize("V,stride", [(4, 4), (32, 40), (300, 384), (1000, 1000), (50277, 50304),
                                      (50277, 50277), (511, 513), (513, 513)])
def test_cdf_bit_exact_vs_oracle(torch, V, stride, bits):
    x = random_logits(6, V, seed=V + bits)
    x[0] = 0  # all-equal row: argmax tie -> index 0
    x[1, V // 2] = 30  # peaked row
    got = _cdf_gpu(torch, x, bits, stride=stride)
    want = coder.cdf_from_logits(x, bits)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("bits", [16, 24])
def test_counts_and_lohi_modes(torch, bits):
    from krunch_b200 import _native as N
    V = 5000
    x = random_logits(9, V, seed=3)
    cdf = coder.cdf_from_logits(x, bits)
    cnt = _cdf_gpu(torch, x, bits, mode=N.KB_CDF_COUNTS)
    assert cnt[:, 0].tolist() == [0] * 9
    assert np.array_equal(np.cumsum(cnt, axis=1), cdf)
    sym = np.random.default_rng(0).integers(0, V, 9)
    lh = _cdf_gpu(torch, x, bits, mode=N.KB_CDF_LOHI, symbols=sym)
    assert np.array_equal(lh, coder.lohi_from_logits(x, sym, bits))


def test_batch_invariance(torch):
    """Rows computed in a batch of R equal rows computed one at a time."""
    x = random_logits(33, 50277, seed=11)
    full = _cdf_gpu(torch, x, 16)
    for r in (0, 7, 32):
        assert np.array_equal(_cdf_gpu(torch, x[r:r + 1], 16), full[r:r + 1])


@pytest.mark.parametrize("bits", [16, 24])
def test_from_probs_bit_exact(torch, bits):
    from krunch_b200.krunch_ac import probs_to_cdf
    from helpers import rand_probs
    p = rand_probs(64, 256, 1)
    got = probs_to_cdf(p, bits)
    assert got.dtype == np.uint32
    assert np.array_equal(got.astype(np.int64), coder.cdf_from_probs(p, bits).astype(np.int64))


@pytest.mark.parametrize("bits", [16, 24])
def test_fused_decode_step_roundtrip(torch, bits):
    """Encode with the oracle from logits; decode on the GPU from the same
    logits with the fused CDF+search+coder kernel, ragged stream lengths."""
    from krunch_b200 import _native as N
    B, T, V, Vp = 4, 40, 3000, 3072
    lens = [40, 1, 25, 0]
    rng = np.random.default_rng(9)
    logits = (rng.standard_normal((T, B, V)) * 3).astype(np.float16)
    sym = rng.integers(0, V, (B, T)).astype(np.int32)
    streams = []
    for b in range(B):
        lh = coder.lohi_from_logits(logits[:lens[b], b], sym[b, :lens[b]], bits)
        streams.append(coder.encode_lohi(lh, bits))
    offs, pos = [], 0
    for s in streams:
        offs.append(pos)
        pos += len(s) + 64
    cat = np.zeros(pos, np.uint8)
    for o, s in zip(offs, streams):
        cat[o:o + len(s)] = np.frombuffer(s, np.uint8)
    inb = torch.from_numpy(cat).cuda()
    offs_t = torch.tensor(offs, dtype=torch.int64, device="cuda")
    st = torch.empty(B * 4, dtype=torch.int32, device="cuda")
    cnt = torch.tensor([[0, n] for n in lens], dtype=torch.int32, device="cuda")
    cur = torch.zeros(B, dtype=torch.int32, device="cuda")
    hist = torch.full((B, T), -1, dtype=torch.int32, device="cuda")
    sp = N.stream_ptr()
    N.call("kb_coder_decode_init", inb.data_ptr(), inb.numel(), offs_t.data_ptr(), st.data_ptr(), B, sp)
    lg = np.zeros((B, Vp), np.float16)
    for t in range(T):
        lg[:, :V] = logits[t]
        x = torch.from_numpy(lg).cuda()
        N.call("kb_decode_logits_step", x.data_ptr(), Vp, B, V, bits, None, 0, inb.data_ptr(),
               inb.numel(),
               offs_t.data_ptr(), st.data_ptr(), cnt.data_ptr(), cur.data_ptr(), hist.data_ptr(),
               T, sp)
    h = hist.cpu().numpy()
    for b in range(B):
        assert h[b, :lens[b]].tolist() == sym[b, :lens[b]].tolist()
        assert (h[b, lens[b]:] == -1).all()
    assert cnt[:, 0].cpu().tolist() == lens


def test_head_gemm_numerators_match_oracle(torch):
    """The head GEMM's softmax numerators and partials == the C oracle's from
    the raw logits, and (lo, hi) from them == (lo, hi) from the raw logits
    == the oracle's."""
    from krunch_b200 import _native as N
    from krunch_b200.model import RWKVModel
    from krunch_b200.synth import random_weights
    m = RWKVModel(random_weights(2, 128, 512, 300, seed=4))
    B, T, V = 3, 9, 300
    tok = torch.from_numpy(np.random.default_rng(3).integers(0, V, (B, T)).astype(np.int32)).cuda()
    raw, num, stats = m.new_logits(B, T), m.new_logits(B, T), m.new_stats(B, T)
    m.forward_window(tok, m.new_state(B), m.new_workspace(B, T), raw)
    m.forward_window(tok, m.new_state(B), m.new_workspace(B, T), num, stats)
    raw_h = raw[:, :V].cpu().numpy()
    e16, ms = coder.softmax_parts(raw_h)
    nsub = ms.shape[1]
    assert np.array_equal(num[:, :nsub * 32].cpu().numpy().view(np.uint16), e16.view(np.uint16))
    assert np.array_equal(stats.cpu().numpy()[:, :nsub].view(np.uint32), ms.view(np.uint32))
    sym = torch.from_numpy(np.random.default_rng(4).integers(0, V, B * T).astype(np.int32)).cuda()
    outs = []
    for x, st, stride in ((num, stats, m.stats_stride), (raw, None, 0)):
        o = torch.empty((B * T, 2), dtype=torch.int32, device="cuda")
        N.call("kb_cdf_rows", x.data_ptr(), m.spec.vocab_pad, B * T, V, 16, N.KB_CDF_LOHI,
               None if st is None else st.data_ptr(), stride, sym.data_ptr(), o.data_ptr(),
               N.stream_ptr())
        outs.append(o.cpu().numpy())
    assert np.array_equal(outs[0], outs[1])
    assert np.array_equal(outs[0].view(np.uint32), coder.lohi_from_logits(raw_h, sym.cpu().numpy(), 16))


@pytest.mark.parametrize("bits", [16, 24])
@pytest.mark.parametrize("V,stride", [(50277, 50304), (1000, 1000), (40, 48), (1001, 1001)])
def test_lohi_from_head_parts_vs_oracle(torch, V, stride, bits):
    """(lo, hi) from stored numerators + partials (the compress path: one warp
    per row, cold subtiles not read) == the oracle's, on flat, peaked,
    all-equal and scaled rows, with symbols at 0, V - 1, the argmax, inside
    and at the edges of subtiles."""
    from krunch_b200 import _native as N
    rng = np.random.default_rng(V + bits)
    x = random_logits(12, V, seed=V * 7 + bits)
    x[0] = 0
    x[1, V // 2] = 30
    x[2] *= 8.0          # peaked: most subtiles cold
    x[3] *= 0.05         # near-flat: every subtile cold at 16 bits
    x[4, :] = -5.0
    x[4, 37 % V] = 4.0
    x = x.astype(np.float16).astype(np.float32)
    e16, ms = coder.softmax_parts(x)
    nsub = ms.shape[1]
    num = np.zeros((12, stride), np.float16)
    num[:, :V] = e16[:, :V]   # (1001: unaligned rows take the one-CTA-per-row kernel)
    st_stride = nsub + (nsub & 1)
    stats = np.zeros((12, st_stride, 2), np.float32)
    stats[:, :nsub] = ms
    sym = rng.integers(0, V, 12)
    sym[:5] = [0, V // 2, int(np.argmax(x[2])), V - 1, 37 % V]
    sym[5] = 31 % V
    sym[6] = 32 % V
    xd = torch.from_numpy(num).cuda()
    sd = torch.from_numpy(stats).cuda()
    yd = torch.from_numpy(sym.astype(np.int32)).cuda()
    o = torch.empty((12, 2), dtype=torch.int32, device="cuda")
    N.call("kb_cdf_rows", xd.data_ptr(), stride, 12, V, bits, N.KB_CDF_LOHI, sd.data_ptr(),
           st_stride, yd.data_ptr(), o.data_ptr(), N.stream_ptr())
    assert np.array_equal(o.cpu().numpy().view(np.uint32), coder.lohi_from_logits(x, sym, bits))
