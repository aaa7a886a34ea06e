"""bf16 model (KB_BF16; BASELINE's bf16 stress runs, the reference's
KRUNCH_BF16 route krunch_ac/cuda/layer_cpp.cpp:224-241): bf16 weights and
GEMM inputs, fp16 residual stream.  GEMMs against a torch fp32 product of the
same bf16 operands, the model against oracle/rwkv.py's bf16 restatement,
packed == stepped bit for bit, and a byte-exact codec round trip."""
import numpy as np
import pytest

from krunch_b200.synth import random_weights

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as t
    return t


def _gemm(torch, A, W, epi, tile_n=0, resid=None, gate=None):
    from krunch_b200 import _native as N
    M, K = A.shape
    Nn = W.shape[0]
    dt = torch.float32 if epi == N.KB_EPI_F32 else (torch.bfloat16 if epi == N.KB_EPI_RELU_SQ
                                                    else torch.float16)
    out = resid.clone() if resid is not None else torch.empty((M, Nn), dtype=dt, device="cuda")
    N.call("kb_gemm_tiled", N.KB_BF16, A.data_ptr(), K, W.data_ptr(), K, M, Nn, K, epi,
           out.data_ptr(), Nn, None if resid is None else out.data_ptr(),
           None if gate is None else gate.data_ptr(), tile_n, N.stream_ptr())
    return out


@pytest.mark.parametrize("epi", range(6))
@pytest.mark.parametrize("M,N,K", [(1, 128, 64), (300, 768, 768), (257, 3072, 768)])
def test_bf16_gemm_vs_torch(torch, epi, M, N, K):
    g = torch.Generator(device="cuda").manual_seed(M + N + K + epi)
    A = (torch.randn((M, K), device="cuda", generator=g) * 0.5).bfloat16()
    W = (torch.randn((N, K), device="cuda", generator=g) * 0.05).bfloat16()
    resid = torch.randn((M, N), device="cuda", generator=g).half()
    gate = torch.rand((M, N), device="cuda", generator=g).half()
    r, gt = (resid if epi >= 4 else None), (gate if epi == 5 else None)
    out = _gemm(torch, A, W, epi, 0, r, gt)
    acc = A.float() @ W.float().t()
    ref = {0: acc, 1: acc, 2: torch.sigmoid(acc), 3: torch.relu(acc) ** 2,
           4: resid.float() + acc, 5: resid.float() + gate.float() * acc}[epi]
    tol = 1e-4 if epi == 0 else (1e-2 if epi == 3 else 2e-2)  # relu^2 written in bf16
    assert (out.float() - ref).abs().max().item() <= tol * max(1.0, ref.abs().max().item())
    for tn in (256, 64, 32):
        assert torch.equal(_gemm(torch, A, W, epi, tn, r, gt), out), tn


def _run(torch, m, tokens, state=None):
    tok = torch.from_numpy(np.ascontiguousarray(tokens, dtype=np.int32)).cuda()
    B, T = tok.shape
    st = m.new_state(B) if state is None else state
    lg = m.new_logits(B, T)
    m.forward_window(tok, st, m.new_workspace(B, T), lg)
    return lg[:, :m.spec.n_vocab].float().view(B, T, -1).cpu().numpy(), st


@pytest.mark.parametrize("shape", [(2, 128, 512, 300), (12, 768, 3072, 50277)])
def test_bf16_model_vs_oracle(torch, shape):
    from krunch_b200.model import RWKVModel
    from oracle import rwkv
    w = random_weights(*shape, seed=3)
    m = RWKVModel(w, wdtype="bf16")
    tok = np.random.default_rng(4).integers(0, shape[3], (2, 5))
    lg, _ = _run(torch, m, tok)
    ref, _ = rwkv.forward(w, tok, wdtype="bf16")
    d = np.abs(lg - ref)
    assert d.max() <= 5e-2 and d.mean() <= 5e-3, (d.max(), d.mean())


def test_bf16_packed_equals_stepped(torch):
    from krunch_b200.model import RWKVModel
    m = RWKVModel(random_weights(2, 128, 512, 300, seed=5), wdtype="bf16")
    tok = np.random.default_rng(1).integers(0, 300, (3, 20))
    packed, st_p = _run(torch, m, tok)
    st = m.new_state(3)
    steps = []
    for t in range(20):
        lg, st = _run(torch, m, tok[:, t:t + 1], st)
        steps.append(lg[:, 0])
    assert np.array_equal(np.stack(steps, 1), packed)
    assert torch.equal(st, st_p)


def test_bf16_codec_roundtrip(torch):
    from krunch_b200.codec import Codec
    from krunch_b200.model import RWKVModel
    from krunch_b200.synth import zipf_tokens
    m = RWKVModel(random_weights(12, 768, 3072, 50277, seed=0), wdtype="bf16")
    codec = Codec(m, cdf_bits=16)
    seqs = list(zipf_tokens((5, 33), seed=2))
    back = codec.decompress_tokens(codec.compress_tokens(seqs), [len(s) for s in seqs])
    for a, b in zip(seqs, back):
        assert np.array_equal(a, b)
