"""kb_forward_window_noalloc: the forward for callers that cannot allocate
device memory (a foreign host under a fixed device-memory budget, or a
caller without a CUDA allocator of its own).  Its activations live in the library's
fixed device array instead of a caller workspace; its output must equal the
regular entry point's.

This file sorts last so that, if it fails, a run stopping at the first
failure has already run every other test.  It creates its own model, so it
also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

from krunch_b200.synth import random_weights

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as t
    return t


def _forward_regular(torch, m, tok, state):
    B, T = tok.shape
    lg = m.new_logits(B, T)
    m.forward_window(tok, state, m.new_workspace(B, T), lg)
    return lg


def _forward_noalloc(torch, m, tok, state):
    from krunch_b200 import _native as N
    B, T = tok.shape
    lg = m.new_logits(B, T)
    N.call("kb_forward_window_noalloc", m.handle, tok.data_ptr(), B, T, state.data_ptr(),
           lg.data_ptr(), N.stream_ptr(m.device))
    return lg


@pytest.mark.parametrize("shape,B,T", [((2, 128, 512, 300), 3, 17), ((12, 768, 3072, 50277), 4, 8)])
def test_noalloc_matches_regular_two_calls(torch, shape, B, T):
    from krunch_b200.model import RWKVModel
    m = RWKVModel(random_weights(*shape, seed=7))
    V = shape[3]
    rng = np.random.default_rng(B * T)
    toks = [torch.from_numpy(rng.integers(0, V, (B, T)).astype(np.int32)).cuda() for _ in range(2)]
    st_a, st_b = m.new_state(B), m.new_state(B)
    for tok in toks:  # two calls in a row; the second continues the state
        want = _forward_regular(torch, m, tok, st_a)
        got = _forward_noalloc(torch, m, tok, st_b)
        torch.cuda.synchronize()
        # the same kernels on the same inputs: identical bits (tolerance 0)
        assert torch.equal(got, want)
        assert torch.equal(st_b, st_a)


def test_noalloc_rejects_oversized_window(torch):
    from krunch_b200 import _native as N
    from krunch_b200.model import RWKVModel
    m = RWKVModel(random_weights(2, 128, 512, 300, seed=1))
    B, T = 64, 512  # far more rows than the fixed scratch holds
    assert m.workspace_bytes(B, T) > N.KB_NOALLOC_SCRATCH_BYTES
    tok = torch.zeros((B, T), dtype=torch.int32, device="cuda")
    st = m.new_state(B)
    lg = m.new_logits(B, T)
    rc = N.load().kb_forward_window_noalloc(m.handle, tok.data_ptr(), B, T, st.data_ptr(),
                                            lg.data_ptr(), ctypes.c_void_p(N.stream_ptr()))
    assert rc == N.KB_ERR_TOO_LARGE
    assert N.load().kb_status_string(rc) == b"request exceeds the fixed no-alloc scratch"
