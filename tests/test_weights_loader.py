"""Checkpoint loader: a state dict in the BlinkDL training layout converts to
the step_ref dictionary (CPU)."""
import numpy as np
import torch

from krunch_b200.synth import random_weights
from krunch_b200.weights import convert_state_dict, load_rwkv4_checkpoint
from oracle import rwkv


def _as_checkpoint(w: dict, ln0_w, ln0_b, emb_raw) -> dict:
    sd = {}
    for k, v in w.items():
        t = torch.from_numpy(np.asarray(v, np.float32).copy())
        if k == "head.weight" or (k.endswith(".weight") and (".att." in k or ".ffn." in k)):
            t = t.t().contiguous()
        elif ".time_" in k:
            t = t.reshape(1, 1, -1) if "mix" in k else t.reshape(-1)
        sd[k] = t.half() if t.ndim == 2 else t
    sd["emb.weight"] = torch.from_numpy(emb_raw).half()
    sd["blocks.0.ln0.weight"] = torch.from_numpy(ln0_w)
    sd["blocks.0.ln0.bias"] = torch.from_numpy(ln0_b)
    return sd


def test_checkpoint_round_trip(tmp_path):
    w = random_weights(2, 128, 512, 300, seed=4)
    rng = np.random.default_rng(0)
    emb_raw = rng.standard_normal((300, 128)).astype(np.float32)
    ln0_w = rng.uniform(0.5, 1.5, 128).astype(np.float32)
    ln0_b = rng.uniform(-0.1, 0.1, 128).astype(np.float32)
    sd = _as_checkpoint(w, ln0_w, ln0_b, emb_raw)
    torch.save(sd, tmp_path / "m.pth")
    got = load_rwkv4_checkpoint(tmp_path / "m.pth")
    assert ".ln0." not in "".join(got)
    e16 = emb_raw.astype(np.float16).astype(np.float32)
    m, v = e16.mean(-1, keepdims=True), e16.var(-1, keepdims=True)
    assert np.allclose(got["emb.weight"], (e16 - m) / np.sqrt(v + 1e-5) * ln0_w + ln0_b, atol=1e-5)
    for k in w:
        if k == "emb.weight":
            continue
        assert got[k].shape == np.asarray(w[k]).shape, k
        tol = 1e-3 if got[k].ndim == 2 else 0
        assert np.abs(got[k] - np.asarray(w[k], np.float32)).max() <= tol * max(1, np.abs(w[k]).max()), k
    # the converted weights run through the oracle forward
    w2 = dict(w, **{"emb.weight": got["emb.weight"]})
    a, _ = rwkv.forward(got, np.array([[1, 2, 3]]))
    b, _ = rwkv.forward(w2, np.array([[1, 2, 3]]))
    assert np.abs(a - b).max() < 2e-2


def test_convert_without_ln0_keeps_emb():
    w = random_weights(1, 128, 512, 300, seed=1)
    sd = {k: np.asarray(v, np.float32) for k, v in w.items()}
    for k in list(sd):
        if k.endswith(".weight") and (".att." in k or ".ffn." in k) or k == "head.weight":
            sd[k] = sd[k].T
    out = convert_state_dict(sd)
    assert np.array_equal(out["emb.weight"], sd["emb.weight"])
