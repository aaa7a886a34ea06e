"""GPU range coder == CPU oracle == reference bytes (reference tests
tests/test_ac_kernel_gpu.py:57-215 shapes and seeds), both CDF totals."""
import json

import numpy as np
import pytest

from helpers import rand_probs, sample_symbols
from oracle import cdf_spec, coder

pytestmark = pytest.mark.gpu
SHAPES = [(1, 4, 0), (8, 32, 1), (256, 256, 2), (1024, 1024, 3), (256, 50277, 4)]


@pytest.fixture(scope="module")
def torch():
    import torch as t
    return t


@pytest.mark.parametrize("bits", [16, 24])
@pytest.mark.parametrize("N,V,seed", SHAPES)
def test_encode_byte_identical(torch, golden_dir, N, V, seed, bits):
    from krunch_b200.krunch_ac import decode, encode
    p = rand_probs(N, V, seed)
    sym = sample_symbols(p, seed)
    cdf = cdf_spec.probs_to_cdf(p, bits)
    bs_gpu = encode(cdf, sym)
    assert bs_gpu == coder.encode(cdf, sym)
    gold = [c for c in json.loads((golden_dir / "coder_cases.json").read_text())
            if c.get("N") == N and c.get("V") == V and c.get("seed") == seed and c["bits"] == bits]
    assert gold and bs_gpu.hex() == gold[0]["bitstream"]
    if N <= 256:
        assert (decode(bs_gpu, cdf) == sym).all()


def test_multi_step_state_persists(torch):
    from krunch_b200 import krunch_ac_cuda as kc
    N_per, V = 100, 256
    rng = np.random.default_rng(42)
    out = torch.zeros(N_per * 3 * 8 + 64, dtype=torch.uint8, device="cuda")
    st = torch.zeros(4, dtype=torch.uint32, device="cuda")
    st[1] = 0xFFFFFFFF
    cdfs, syms = [], []
    for i in range(3):
        c = cdf_spec.probs_to_cdf(rand_probs(N_per, V, i), 24)
        s = rng.integers(0, V, N_per).astype(np.int32)
        kc.encode_step(torch.from_numpy(c.astype(np.int32)).cuda(), torch.from_numpy(s).cuda(), out, st)
        cdfs.append(c)
        syms.append(s)
    kc.encode_finalize(out, st)
    n = (int(st[3].item()) + 7) // 8
    assert out[:n].cpu().numpy().tobytes() == coder.encode(np.concatenate(cdfs), np.concatenate(syms))


@pytest.mark.parametrize("B,N,V,seed", [(2, 16, 32, 7), (4, 64, 256, 8), (8, 256, 1024, 9),
                                        (3, 1024, 50277, 10)])
def test_decode_step_batched_roundtrip(torch, B, N, V, seed):
    from krunch_b200 import krunch_ac_cuda as kc
    streams, cdfs, syms = [], [], []
    for b in range(B):
        p = rand_probs(N, V, seed + b)
        s = sample_symbols(p, seed + b)
        c = cdf_spec.probs_to_cdf(p, 24)
        streams.append(coder.encode(c, s))
        cdfs.append(c)
        syms.append(s)
    offs, pos = [], 0
    for bs in streams:
        offs.append(pos)
        pos += len(bs) + 64
    cat = bytearray(pos)
    for o, bs in zip(offs, streams):
        cat[o:o + len(bs)] = bs
    inb = torch.frombuffer(bytearray(cat), dtype=torch.uint8).clone().cuda()
    offs_t = torch.tensor(offs, dtype=torch.int32, device="cuda")
    st = torch.zeros(B * 4, dtype=torch.uint32, device="cuda")
    kc.decode_init_batched(inb, offs_t, st)
    out = torch.empty(B, dtype=torch.int32, device="cuda")
    dec = np.empty((B, N), np.int32)
    all_cdfs = torch.from_numpy(np.stack(cdfs).astype(np.int32)).cuda()  # [B, N, V+1]
    for t in range(N):
        kc.decode_step_batched(all_cdfs[:, t].contiguous(), inb, offs_t, st, out)
        dec[:, t] = out.cpu().numpy()
    for b in range(B):
        assert (dec[b] == syms[b]).all()


def test_encode_step_batched_matches_oracle(torch):
    from krunch_b200 import krunch_ac_cuda as kc
    B, N, V = 5, 40, 300
    cdfs = [cdf_spec.probs_to_cdf(rand_probs(N, V, 50 + b), 24) for b in range(B)]
    syms = [sample_symbols(rand_probs(N, V, 50 + b), 50 + b) for b in range(B)]
    stride = N * 4 + 64
    out = torch.zeros(B * stride, dtype=torch.uint8, device="cuda")
    offs = torch.arange(B, dtype=torch.int32, device="cuda") * stride
    st = torch.zeros((B, 4), dtype=torch.uint32, device="cuda")
    st[:, 1] = 0xFFFFFFFF
    c_all = torch.from_numpy(np.stack(cdfs).astype(np.int32)).cuda()
    s_all = torch.from_numpy(np.stack(syms)).cuda()
    for t in range(N):
        kc.encode_step_batched(c_all[:, t].contiguous(), s_all[:, t].contiguous(), out, offs, st)
    kc.encode_finalize_batched(out, offs, st)
    h = out.cpu().numpy()
    nb = st[:, 3].cpu().numpy().astype(np.int64)
    for b in range(B):
        n = (int(nb[b]) + 7) // 8
        assert h[b * stride:b * stride + n].tobytes() == coder.encode(cdfs[b], syms[b])


@pytest.mark.parametrize("bits", [16, 24])
def test_encode_lohi_windows_and_ragged(torch, bits):
    """Lane-per-stream encode over two windows with ragged stream lengths."""
    from krunch_b200 import _native as N
    B, T, V = 6, 50, 700
    lens = np.array([50, 1, 17, 0, 49, 33])
    rng = np.random.default_rng(5)
    logits = rng.standard_normal((B, T, V)).astype(np.float16)
    sym = rng.integers(0, V, (B, T)).astype(np.int32)
    lohi = coder.lohi_from_logits(logits.reshape(-1, V), sym.reshape(-1), bits).reshape(B, T, 2)
    cap = 512
    out = torch.zeros(B * cap, dtype=torch.uint8, device="cuda")
    offs = torch.arange(B, dtype=torch.int64, device="cuda") * cap
    st = torch.empty(B * 4, dtype=torch.int32, device="cuda")
    s = N.stream_ptr()
    N.call("kb_coder_encode_init", st.data_ptr(), B, s)
    for off, tw in ((0, 20), (20, 30)):
        w = torch.from_numpy(np.ascontiguousarray(lohi[:, off:off + tw]).view(np.int32)).cuda()
        nv = torch.from_numpy(np.clip(lens - off, 0, tw).astype(np.int32)).cuda()
        N.call("kb_coder_encode_lohi", w.data_ptr(), B, tw, nv.data_ptr(), bits, out.data_ptr(),
               out.numel(), offs.data_ptr(), st.data_ptr(), s)
    N.call("kb_coder_encode_finalize", out.data_ptr(), out.numel(), offs.data_ptr(), st.data_ptr(), B, s)
    h = out.cpu().numpy()
    nb = st.view(B, 4)[:, 3].cpu().numpy()
    for b in range(B):
        n = (int(nb[b]) + 7) // 8
        assert h[b * cap:b * cap + n].tobytes() == coder.encode_lohi(lohi[b, :lens[b]], bits)
