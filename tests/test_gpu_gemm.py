"""GEMM + fused epilogues against a plain PyTorch fp32 reference, and the
M-invariance contract (reference scripts/test_det_matmul_tc_mw.py:20-39:
a row's bits do not depend on M)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as t
    return t


def _gemm(torch, A, W, epi, resid=None, gate=None, out_dtype=None):
    from krunch_b200 import _native as N
    M, K = A.shape
    Nn = W.shape[0]
    dt = torch.float32 if epi == N.KB_EPI_F32 else torch.float16
    out = resid.clone() if resid is not None else torch.empty((M, Nn), dtype=dt, device="cuda")
    N.call("kb_gemm", N.KB_F16, A.data_ptr(), K, W.data_ptr(), K, M, Nn, K, epi, out.data_ptr(),
           Nn, None if resid is None else out.data_ptr(), None if gate is None else gate.data_ptr(),
           N.stream_ptr())
    return out


def _ref(torch, A, W, epi, resid=None, gate=None):
    from krunch_b200 import _native as N
    acc = A.float() @ W.float().t()
    if epi == N.KB_EPI_SIGMOID:
        return torch.sigmoid(acc)
    if epi == N.KB_EPI_RELU_SQ:
        return torch.relu(acc) ** 2
    if epi == N.KB_EPI_RESID:
        return resid.float() + acc
    if epi == N.KB_EPI_GATE_RESID:
        return resid.float() + gate.float() * acc
    return acc


@pytest.mark.parametrize("epi", range(6))
@pytest.mark.parametrize("M,N,K", [(1, 128, 64), (77, 256, 192), (300, 768, 768), (1000, 384, 3072)])
def test_gemm_epilogues_vs_torch_fp32(torch, epi, M, N, K):
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N + K + epi)
    A = (torch.randn((M, K), device="cuda", generator=g) * 0.5).half()
    W = (torch.randn((N, K), device="cuda", generator=g) * 0.05).half()
    resid = torch.randn((M, N), device="cuda", generator=g).half()
    gate = torch.rand((M, N), device="cuda", generator=g).half()
    out = _gemm(torch, A, W, epi, resid if epi >= 4 else None, gate if epi == 5 else None)
    ref = _ref(torch, A, W, epi, resid, gate)
    tol = 1e-4 if epi == 0 else 2e-2
    err = (out.float() - ref).abs().max().item()
    assert err <= tol * max(1.0, ref.abs().max().item()), err


def test_m_invariance(torch):
    from krunch_b200 import _native as N
    g = torch.Generator(device="cuda").manual_seed(1)
    K, Nn = 768, 768
    A = (torch.randn((1000, K), device="cuda", generator=g)).half()
    W = (torch.randn((Nn, K), device="cuda", generator=g) * 0.03).half()
    full = _gemm(torch, A, W, N.KB_EPI_F32)
    for M in (1, 16, 64, 128, 129, 256, 999):
        part = _gemm(torch, A[:M].contiguous(), W, N.KB_EPI_F32)
        assert torch.equal(part, full[:M]), M
    rows = A[[5, 900, 3]].contiguous()
    assert torch.equal(_gemm(torch, rows, W, N.KB_EPI_F32), full[[5, 900, 3]])


def _gemm_tiled(torch, A, W, epi, tile_n, resid=None, gate=None, dtype=None):
    from krunch_b200 import _native as N
    dtype = N.KB_F16 if dtype is None else dtype
    M, K = A.shape
    Nn = W.shape[0]
    dt = torch.float32 if epi == N.KB_EPI_F32 else torch.float16
    out = resid.clone() if resid is not None else torch.empty((M, Nn), dtype=dt, device="cuda")
    N.call("kb_gemm_tiled", dtype, A.data_ptr(), K, W.data_ptr(), K, M, Nn, K, epi,
           out.data_ptr(), Nn, None if resid is None else out.data_ptr(),
           None if gate is None else gate.data_ptr(), tile_n, N.stream_ptr())
    return out


@pytest.mark.parametrize("epi", range(6))
@pytest.mark.parametrize("M,N,K", [(256, 768, 768), (33, 3072, 768), (300, 768, 3072)])
def test_tile_width_invariance(torch, epi, M, N, K):
    """Every output tile width gives the same bits (the decoder's small-M
    launches use narrow tiles, the encoder's packed launches 256 wide)."""
    g = torch.Generator(device="cuda").manual_seed(M + N + K + epi)
    A = (torch.randn((M, K), device="cuda", generator=g) * 0.5).half()
    W = (torch.randn((N, K), device="cuda", generator=g) * 0.05).half()
    resid = torch.randn((M, N), device="cuda", generator=g).half()
    gate = torch.rand((M, N), device="cuda", generator=g).half()
    r, gt = (resid if epi >= 4 else None), (gate if epi == 5 else None)
    want = _gemm_tiled(torch, A, W, epi, 256, r, gt)
    for tn in (128, 64, 32, 0):
        assert torch.equal(_gemm_tiled(torch, A, W, epi, tn, r, gt), want), tn


@pytest.mark.parametrize("epi", range(6))
@pytest.mark.parametrize("M,N,K", [(256, 768, 768), (1000, 3072, 768), (300, 768, 3072),
                                   (40000, 768, 768)])
@pytest.mark.parametrize("bf16", [False, True])
def test_cta_pair_tiles_bit_identical(torch, epi, M, N, K, bf16):
    """The CTA-pair kernel (256 x 256 tiles, cta_group::2 MMAs; the library's
    choice for large M) gives the bits of the single-CTA kernel, including
    for M not a multiple of 256 and for more tiles than resident pairs."""
    from krunch_b200 import _native as N_
    g = torch.Generator(device="cuda").manual_seed(M + N + K + epi + 11)
    dt = torch.bfloat16 if bf16 else torch.float16
    A = (torch.randn((M, K), device="cuda", generator=g) * 0.5).to(dt)
    W = (torch.randn((N, K), device="cuda", generator=g) * 0.05).to(dt)
    resid = torch.randn((M, N), device="cuda", generator=g).half()
    gate = torch.rand((M, N), device="cuda", generator=g).half()
    r, gt = (resid if epi >= 4 else None), (gate if epi == 5 else None)
    kind = N_.KB_BF16 if bf16 else N_.KB_F16
    want = _gemm_tiled(torch, A, W, epi, 256, r, gt, kind)
    got = _gemm_tiled(torch, A, W, epi, N_.KB_TILE_PAIR, r, gt, kind)
    assert torch.equal(got, want)
    if epi == 0:
        ref = A.float() @ W.float().t()
        assert (got - ref).abs().max().item() <= 1e-4 * max(1.0, ref.abs().max().item())
