"""The reference's import names and Python contracts on the GPU:

* ``krunch`` / ``krunch_ac`` / ``krunch_ac_cuda`` resolve to this build;
* ``krunch_ac_cuda.rwkv4_layer_step_cpp[_t1]`` (layer_cpp.cpp:294-307,
  456-637) with the reference's tensor layout gives the bits of
  ``kb_layer_forward`` (the layer of ``kb_forward_window``) and, followed by
  the final LayerNorm and ``det_matmul`` head, logits within 2e-2 of the
  oracle (production WKV, the convention of the reference's layer);
* ``batched_rwkv4.init_state_batched`` / ``forward_batched`` keep the 5*L
  list contract (batched_rwkv4.py:60-82, 175-262);
* ``cpp_path`` packed windows == stepped batched, bit for bit
  (scripts/test_full_model_packed_vs_stepped.py:77-110), and its CDFs equal
  the oracle's."""

import numpy as np
import pytest

from krunch_b200.synth import random_weights

pytestmark = pytest.mark.gpu
LOGIT_TOL = 2e-2


@pytest.fixture(scope="module")
def torch():
    import torch as t
    return t


def _fp16_exact(w):
    """Round every vector to fp16 (the reference keeps LN and mixes in fp16)
    so both layouts see the same values."""
    out = dict(w)
    for k, v in w.items():
        if v.ndim == 1 and "time_decay" not in k and "time_first" not in k:
            out[k] = v.astype(np.float16).astype(np.float32)
    return out


def test_reference_import_names(torch):
    import krunch.batched_rwkv4
    import krunch.chunking
    import krunch.cpp_path
    import krunch.inference
    import krunch_ac
    import krunch_ac.cdf
    import krunch_ac_cuda
    import krunch_b200
    from oracle import coder
    assert krunch.inference.engine.__class__.__module__ == "krunch_b200.inference"
    assert krunch.inference.HEADER_SIZE == 37 and krunch.inference.BOS_TOKEN == 0
    assert krunch_ac_cuda.__name__ == "krunch_b200.krunch_ac_cuda"
    assert krunch_ac.cdf.CDF_PRECISION == 24 and krunch_b200 is not None
    # encode_cpu / decode_cpu: the reference's signatures and bytes (on the GPU)
    rng = np.random.default_rng(3)
    p = rng.random((40, 64)).astype(np.float32)
    p /= p.sum(1, keepdims=True)
    cdf = krunch_ac.probs_to_cdf(p)
    cdf = cdf.cpu().numpy() if hasattr(cdf, "cpu") else np.asarray(cdf)
    sym = rng.integers(0, 64, 40).astype(np.int32)
    bs = krunch_ac.encode_cpu(cdf, sym)
    assert bs == coder.encode(cdf, sym)
    assert np.array_equal(krunch_ac.decode_cpu(bs, cdf), sym)


def _ref_layer_tensors(torch, w, i, dev, decay):
    """The 18 tensors of cpp_path.init_weights (cpp_path.py:59-78): fp16
    LN / mixes, fp32 time_decay as the rwkv loader leaves it (-exp(raw)) and
    time_first, matrices [in, out] fp16."""
    b, att, ffn = f"blocks.{i}.", f"blocks.{i}.att.", f"blocks.{i}.ffn."
    h = lambda k: torch.from_numpy(w[k]).to(dev, torch.float16)  # noqa: E731
    f = lambda a: torch.as_tensor(a).to(dev, torch.float32)  # noqa: E731
    return [h(b + "ln1.weight"), h(b + "ln1.bias"), h(att + "time_mix_k"), h(att + "time_mix_v"),
            h(att + "time_mix_r"), -decay, f(w[att + "time_first"]),
            h(att + "key.weight"), h(att + "value.weight"), h(att + "receptance.weight"),
            h(att + "output.weight"), h(b + "ln2.weight"), h(b + "ln2.bias"),
            h(ffn + "time_mix_k"), h(ffn + "time_mix_r"), h(ffn + "key.weight"),
            h(ffn + "value.weight"), h(ffn + "receptance.weight")]


@pytest.mark.parametrize("B,T", [(3, 7), (1, 1)])
def test_layer_step_cpp_matches_layer_forward(torch, B, T):
    import krunch_ac_cuda
    from krunch_b200 import _native as N
    from krunch_b200.model import RWKVModel
    from oracle import rwkv
    w = _fp16_exact(random_weights(2, 128, 512, 300, seed=12))
    m = RWKVModel(w, wkv="production")
    dev = m.device
    ids = np.random.default_rng(4).integers(0, 300, (B, T)).astype(np.int32)
    x0 = m.emb[torch.from_numpy(ids).long().to(dev)].reshape(B * T, -1).contiguous()

    # chain A: kb_layer_forward on the model handle
    xa = x0.clone()
    st = m.new_state(B)
    ws = m.new_workspace(B, T)
    for i in range(2):
        N.call("kb_layer_forward", m.handle, i, xa.data_ptr(), B, T, st[i].data_ptr(),
               ws.data_ptr(), ws.numel(), N.stream_ptr(dev))

    # chain B: the reference's call with the reference's tensors and state
    Cm = 128
    xb = x0.view(B, T, Cm).clone()
    states = []
    for i in range(2):
        td = torch.from_numpy(w[f"blocks.{i}.att.time_decay"]).to(dev)
        decay = torch.empty_like(td)
        N.call("kb_prepare_decay", td.data_ptr(), decay.data_ptr(), td.numel(), N.stream_ptr(dev))
        s = [torch.zeros(B, Cm, dtype=torch.float16, device=dev),
             torch.zeros(B, Cm, dtype=torch.float32, device=dev),
             torch.zeros(B, Cm, dtype=torch.float32, device=dev),
             torch.full((B, Cm), -1e30, dtype=torch.float32, device=dev),
             torch.zeros(B, Cm, dtype=torch.float16, device=dev)]
        fn = krunch_ac_cuda.rwkv4_layer_step_cpp_t1 if (B, T) == (1, 1) else \
            krunch_ac_cuda.rwkv4_layer_step_cpp
        xb = fn(xb, *s, *_ref_layer_tensors(torch, w, i, dev, decay))
        states.append(s)
    assert torch.equal(xb.reshape(B * T, Cm), xa)
    for i in range(2):
        for j in range(5):
            assert torch.equal(states[i][j].float(), st[i, j]), (i, j)

    # final LayerNorm + det_matmul head vs the oracle
    xn = torch.nn.functional.layer_norm(xb.reshape(B * T, Cm).float(), (Cm,),
                                        torch.from_numpy(w["ln_out.weight"]).to(dev),
                                        torch.from_numpy(w["ln_out.bias"]).to(dev)).half()
    lg = krunch_ac_cuda.det_matmul(xn.contiguous(), torch.from_numpy(w["head.weight"]).to(dev).half())
    ref, _ = rwkv.forward(w, ids, wkv="production")
    assert np.abs(lg.float().cpu().numpy().reshape(B, T, -1) - ref).max() <= LOGIT_TOL


def test_forward_batched_list_contract(torch):
    from krunch_b200.batched_rwkv4 import forward_batched, init_state_batched
    from krunch_b200.model import RWKVModel
    from oracle import rwkv
    w = random_weights(2, 128, 512, 300, seed=13)
    m = RWKVModel(w)
    tok = np.random.default_rng(5).integers(0, 300, (3, 10))
    state = init_state_batched(m, 3)
    assert len(state) == 10
    assert [t.dtype for t in state[:5]] == [torch.float16, torch.float32, torch.float32,
                                            torch.float32, torch.float16]
    assert float(state[3].max()) == torch.tensor(-1e30).item()
    same = state
    a, state = forward_batched(m, tok[:, :4].tolist(), state)
    assert state is same and state[0].dtype == torch.float16
    b, state = forward_batched(m, torch.as_tensor(tok[:, 4:]).cuda(), state, full_output=True)
    last, _ = forward_batched(m, tok[:, :4].tolist(), init_state_batched(m, 3), full_output=False)
    assert a.dtype == torch.float16 and a.shape == (3, 4, 300) and last.shape == (3, 300)
    assert torch.equal(last, a[:, -1])
    got = torch.cat([a, b], 1).float().cpu().numpy()
    # one window on a stacked state gives the same bits
    one, st2 = forward_batched(m, torch.as_tensor(tok).cuda(), m.new_state(3))
    assert np.array_equal(one.float().cpu().numpy(), got)
    ref, ref_st = rwkv.forward(w, tok)
    assert np.abs(got - ref).max() <= LOGIT_TOL
    for i in range(10):
        assert np.abs(state[i].float().cpu().numpy() - ref_st[i]).max() <= 2e-2 * max(
            1.0, np.abs(ref_st[i]).max()), i


def test_cpp_path_packed_equals_stepped_and_cdf(torch):
    from krunch_b200 import cpp_path
    from oracle import coder
    w = random_weights(2, 128, 512, 300, seed=14)
    m = cpp_path.init_weights(w)
    assert cpp_path.init_weights(w) is m
    ids = np.random.default_rng(6).integers(0, 300, 24)
    st = cpp_path.fresh_state(m)
    packed = torch.cat([cpp_path.forward_packed_window(m, ids, st, 0, 10),
                        cpp_path.forward_packed_window(m, ids, st, 10, 14)])
    sb = cpp_path.fresh_state_batched(m, 2)
    steps = []
    for t in range(24):
        steps.append(cpp_path.forward_stepped_batched(m, [int(ids[t]), int(ids[t])], sb))
    stepped = torch.stack(steps, 1)
    assert torch.equal(stepped[0], packed) and torch.equal(stepped[1], packed)
    for j in range(5):
        assert torch.equal(st[j][0], sb[j][0][:1]) and torch.equal(sb[j][0][0], sb[j][0][1])
    s1 = cpp_path.fresh_state(m)
    one = cpp_path.forward_stepped(m, int(ids[0]), s1)
    assert torch.equal(one, packed[0])
    cdf = cpp_path.softmax_cdfs_per_row(packed)
    want = coder.cdf_from_logits(packed.cpu().numpy(), 24)
    assert np.array_equal(cdf.cpu().numpy(), want)
    assert torch.equal(cpp_path.softmax_cdf_one_row(packed[5]), cdf[5])
    assert cpp_path.compute_decompress_batch(5) == 5


def test_layer_step_cache_sees_in_place_edits(torch):
    """The reference-named layer step caches its converted weights; an
    in-place edit of an input tensor is picked up, a repeated call reuses
    the entry."""
    import krunch_ac_cuda
    from krunch_b200 import _native as N
    w = _fp16_exact(random_weights(1, 128, 512, 300, seed=15))
    dev = torch.device("cuda")
    td = torch.from_numpy(w["blocks.0.att.time_decay"]).to(dev)
    decay = torch.empty_like(td)
    N.call("kb_prepare_decay", td.data_ptr(), decay.data_ptr(), td.numel(), N.stream_ptr(dev))
    layer = _ref_layer_tensors(torch, w, 0, dev, decay)
    x = (torch.randn((2, 5, 128), device=dev) * 0.1).half()

    def run():
        s = [torch.zeros(2, 128, dtype=torch.float16, device=dev),
             torch.zeros(2, 128, device=dev), torch.zeros(2, 128, device=dev),
             torch.full((2, 128), -1e30, device=dev),
             torch.zeros(2, 128, dtype=torch.float16, device=dev)]
        return krunch_ac_cuda.rwkv4_layer_step_cpp(x, *s, *layer)

    krunch_ac_cuda.clear_layer_graph_cache()
    a = run()
    b = run()
    assert torch.equal(a, b) and len(krunch_ac_cuda._LAYER_CACHE) == 1
    layer[10].mul_(2.0)  # Ow, in place
    c = run()
    assert len(krunch_ac_cuda._LAYER_CACHE) == 2 and not torch.equal(a, c)
    krunch_ac_cuda.clear_layer_graph_cache()
    assert torch.equal(run(), c)


def test_reference_bench_names(torch):
    """det_matmul_bf16 / det_matmul_tc_3way_async / phase-time readers under
    the reference's names (layer_cpp.cpp:825-960) against torch fp32."""
    import krunch_ac_cuda
    g = torch.Generator(device="cuda").manual_seed(4)
    x = (torch.randn((70, 768), device="cuda", generator=g) * 0.5)
    W = (torch.randn((768, 300), device="cuda", generator=g) * 0.05)
    ref = x @ W
    yb = krunch_ac_cuda.det_matmul_bf16(x.bfloat16(), W.bfloat16())
    assert yb.dtype == torch.bfloat16 and yb.shape == (70, 300)
    refb = x.bfloat16().float() @ W.bfloat16().float()
    assert (yb.float() - refb).abs().max().item() <= 2e-2 * max(1.0, refb.abs().max().item())
    krunch_ac_cuda.reset_phase_times()
    ys = krunch_ac_cuda.det_matmul_tc_3way_async(x.half(), x.half(), x.half(), W.half(),
                                                 W.half(), W.half(), torch.float32)
    times = krunch_ac_cuda.read_phase_times()
    assert len(ys) == 3 and all(torch.equal(ys[0], y) for y in ys) and ys[0].dtype == torch.float32
    assert (ys[0] - ref).abs().max().item() <= 2e-2
    assert times["call_count"] == 3 and times["gemm"] > 0
