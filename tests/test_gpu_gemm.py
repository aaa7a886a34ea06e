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


@pytest.mark.parametrize("dtype", ["f16", "bf16", "i8"])
@pytest.mark.parametrize("M,tile", [(1, 0), (300, 0), (300, 64), (9000, 0), (70000, 0),
                                     (70000, 512)])
def test_grouped_kvr_equals_three_launches(torch, dtype, M, tile):
    """kb_gemm_kvr (one launch: k, v fp32, r = sigmoid fp16; the reference's
    det_matmul_tc_3way_async.cu:50-251) gives the bits of three single
    launches, on single-CTA and CTA-pair tilings."""
    from krunch_b200 import _native as N
    C = 768
    g = torch.Generator(device="cuda").manual_seed(M + tile)
    i8 = dtype == "i8"
    if i8:
        A = [torch.randint(-127, 128, (M, C), device="cuda", dtype=torch.int8, generator=g)
             for _ in range(3)]
        W = [torch.randint(-127, 128, (C, C), device="cuda", dtype=torch.int8, generator=g)
             for _ in range(3)]
        sa = [torch.rand(M, device="cuda", generator=g) * 1e-2 for _ in range(3)]
        sw = [(torch.rand(C, device="cuda", generator=g) * 1e-2).half() for _ in range(3)]
    else:
        dt = torch.bfloat16 if dtype == "bf16" else torch.float16
        A = [(torch.randn((M, C), device="cuda", generator=g) * 0.5).to(dt) for _ in range(3)]
        W = [(torch.randn((C, C), device="cuda", generator=g) * 0.05).to(dt) for _ in range(3)]
        sa, sw = [None] * 3, [None] * 3
    kind = {"f16": N.KB_F16, "bf16": N.KB_BF16, "i8": N.KB_I8}[dtype]
    k = torch.empty((M, C), device="cuda")
    v = torch.empty((M, C), device="cuda")
    r = torch.empty((M, C), device="cuda", dtype=torch.float16)
    p = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    N.call("kb_gemm_kvr", kind, A[0].data_ptr(), A[1].data_ptr(), A[2].data_ptr(), C,
           p(sa[0]), p(sa[1]), p(sa[2]), W[0].data_ptr(), W[1].data_ptr(), W[2].data_ptr(), C,
           p(sw[0]), p(sw[1]), p(sw[2]), M, C, C, k.data_ptr(), v.data_ptr(), r.data_ptr(), C,
           tile, N.stream_ptr())
    for j, (out, epi) in enumerate(((k, N.KB_EPI_F32), (v, N.KB_EPI_F32), (r, N.KB_EPI_SIGMOID))):
        ref = torch.empty_like(out)
        if i8:
            N.call("kb_gemm_i8", A[j].data_ptr(), C, sa[j].data_ptr(), W[j].data_ptr(), C,
                   sw[j].data_ptr(), M, C, C, epi, ref.data_ptr(), C, None, None, tile,
                   N.stream_ptr())
        else:
            N.call("kb_gemm_tiled", kind, A[j].data_ptr(), C, W[j].data_ptr(), C, M, C, C, epi,
                   ref.data_ptr(), C, None, None, tile, N.stream_ptr())
        assert torch.equal(out, ref), (dtype, M, tile, j)
