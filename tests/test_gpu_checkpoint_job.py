"""The real-weights loader and the multi-part job on the GPU.

* A `.pth` checkpoint in the BlinkDL training layout (the file the reference
  loads through rwkv.model.RWKV, krunch/inference.py:181-194; ln0 present,
  Linear weights [out, in], fp16 matrices) loads through weights.py and runs
  through the kernels within 2e-2 of the oracle on the same converted
  weights, directly and as the engine's `pile169m` family.
* A 2-part compress job (krunch/job.py:73-231: byte-range workers, then the
  finalize stitch) through the real GPU codec gives the bytes of a
  single-process compress of the whole input, and the 2-part decompress job
  gives the input back."""
import os

import numpy as np
import pytest
import torch

from krunch_b200.synth import markov_text, random_weights

pytestmark = pytest.mark.gpu
LOGIT_TOL = 2e-2


def _write_checkpoint(path, w, seed=0):
    rng = np.random.default_rng(seed)
    C = w["emb.weight"].shape[1]
    sd = {}
    for k, v in w.items():
        t = torch.from_numpy(np.asarray(v, np.float32).copy())
        if k == "head.weight" or (k.endswith(".weight") and (".att." in k or ".ffn." in k)):
            t = t.t().contiguous()
        elif ".time_" in k:
            t = t.reshape(1, 1, -1) if "mix" in k else t.reshape(-1)
        sd[k] = t.half() if t.ndim == 2 else t
    sd["emb.weight"] = torch.from_numpy(rng.standard_normal(w["emb.weight"].shape).astype(np.float32)).half()
    sd["blocks.0.ln0.weight"] = torch.from_numpy(rng.uniform(0.5, 1.5, C).astype(np.float32))
    sd["blocks.0.ln0.bias"] = torch.from_numpy(rng.uniform(-0.1, 0.1, C).astype(np.float32))
    torch.save(sd, path)


def test_checkpoint_through_kernels_vs_oracle(tmp_path):
    from krunch_b200.model import RWKVModel
    from krunch_b200.weights import load_rwkv4_checkpoint
    from oracle import rwkv
    _write_checkpoint(tmp_path / "m.pth", random_weights(2, 128, 512, 300, seed=21))
    w = load_rwkv4_checkpoint(tmp_path / "m.pth")
    m = RWKVModel(w)
    tok = np.random.default_rng(3).integers(0, 300, (2, 17)).astype(np.int32)
    t = torch.from_numpy(tok).cuda()
    lg = m.new_logits(2, 17)
    m.forward_window(t, m.new_state(2), m.new_workspace(2, 17), lg)
    got = lg[:, :300].float().view(2, 17, -1).cpu().numpy()
    ref, _ = rwkv.forward(w, tok)
    assert np.abs(got - ref).max() <= LOGIT_TOL


def test_engine_loads_pile169m_family(tmp_path, monkeypatch):
    from krunch_b200 import inference
    from krunch_b200.weights import PILE_169M_FILE
    _write_checkpoint(tmp_path / PILE_169M_FILE, random_weights(2, 128, 512, 300, seed=22), seed=1)
    monkeypatch.setenv("KRUNCH_MODEL_DIR", str(tmp_path))
    monkeypatch.setenv("KRUNCH_MODEL", "pile169m")
    monkeypatch.setenv("KRUNCH_TOKENIZER", "byte")
    monkeypatch.setenv("KRUNCH_CDF_BITS", "16")
    monkeypatch.setattr(inference, "_MODEL_CACHE", {})
    e = inference.InferenceEngine()
    e.load()
    assert e.cfg.family == "pile169m" and e.codec.model.spec.n_embd == 128
    chunks = [markov_text(2500, seed=9), "pile ✓ ".encode() * 30]
    assert e.decompress_chunks_batched(e.compress_chunks_batched(chunks)) == chunks


def test_two_part_job_matches_single_process(tmp_path, monkeypatch):
    from krunch_b200 import cli, inference, job
    monkeypatch.setenv("KRUNCH_MODEL", "tiny")
    monkeypatch.setenv("KRUNCH_TOKENIZER", "byte")
    monkeypatch.setenv("KRUNCH_CDF_BITS", "16")
    monkeypatch.setenv("KRUNCH_CHUNK_SIZE", "4096")
    monkeypatch.setattr(inference, "engine", inference.InferenceEngine())
    monkeypatch.setattr(cli, "engine", inference.engine, raising=False)
    raw = markov_text(30_000, seed=12)  # ASCII: part boundaries never split a character
    src = tmp_path / "in.txt"
    src.write_bytes(raw)
    blob = tmp_path / "out.krunch"
    base = {"KRUNCH_INPUT_URL": str(src), "KRUNCH_OUTPUT_URL": str(blob),
            "KRUNCH_PART_COUNT": "2", "KRUNCH_INPUT_LEN": str(len(raw))}
    for i in range(2):
        job.run({**base, "KRUNCH_MODE": "compress", "KRUNCH_PART_INDEX": str(i)})
    job.run({**base, "KRUNCH_MODE": "finalize", "KRUNCH_FINALIZE_OF": "compress"})
    single = cli.compress_bytes(raw)
    assert blob.read_bytes() == single
    out = tmp_path / "back.txt"
    dbase = {"KRUNCH_INPUT_URL": str(blob), "KRUNCH_OUTPUT_URL": str(out), "KRUNCH_PART_COUNT": "2"}
    for i in range(2):
        job.run({**dbase, "KRUNCH_MODE": "decompress", "KRUNCH_PART_INDEX": str(i)})
    job.run({**dbase, "KRUNCH_MODE": "finalize", "KRUNCH_FINALIZE_OF": "decompress"})
    assert out.read_bytes() == raw
