"""End-to-end byte-exact round trips through the codec, the engine and the
CLI, and compressed size against the CPU oracle pipeline (BASELINE: within
0.5%)."""
import os
import subprocess
import sys

import numpy as np
import pytest

from krunch_b200.synth import markov_text, random_weights

pytestmark = pytest.mark.gpu
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(REPO, "tests", "golden")


@pytest.fixture(scope="module")
def torch():
    import torch as t
    return t


@pytest.mark.parametrize("bits", [16, 24])
def test_codec_roundtrip_ragged(torch, bits):
    from krunch_b200.codec import Codec
    from krunch_b200.model import RWKVModel
    m = RWKVModel(random_weights(2, 128, 512, 300, seed=1))
    rng = np.random.default_rng(bits)
    seqs = [rng.integers(0, 300, n).astype(np.int32) for n in (1, 2, 57, 300, 129)]
    codec = Codec(m, cdf_bits=bits)
    streams = codec.compress_tokens(seqs)
    # a different window size and batch grouping give the same bytes
    os.environ["KRUNCH_FORWARD_BATCH"] = "16"
    try:
        again = Codec(m, cdf_bits=bits).compress_tokens(seqs, max_batch=2)
    finally:
        del os.environ["KRUNCH_FORWARD_BATCH"]
    assert again == streams
    back = codec.decompress_tokens(streams, [len(s) for s in seqs])
    for a, b in zip(seqs, back):
        assert np.array_equal(a, b)
    back1 = codec.decompress_tokens(streams[2:3], [57])
    assert np.array_equal(back1[0], seqs[2])


_ORACLE_LOGITS = {}


def _peaked():
    """Peaked RWKV-4-169M (head x8) and 4 x 512 tokens sampled from it
    (tests/golden/make_peaked.py): the model is the streams' generator, so
    its code length is informative (~5-7 bits/token, not the ~16 of the
    near-uniform random init) and a wrong model pays a KL excess."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_peaked", os.path.join(GOLDEN, "make_peaked.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.peaked_weights(), list(np.load(os.path.join(GOLDEN, "peaked_169m_tokens.npy")))


def test_compress_batches_pipelined_equals_single(torch):
    """Codec.compress_batches (batch i+1 prepared and enqueued while batch i
    runs, results through pinned memory) yields each batch's bytes exactly
    as compress_tokens does, in order."""
    from krunch_b200.codec import Codec
    from krunch_b200.model import RWKVModel
    codec = Codec(RWKVModel(random_weights(2, 128, 512, 300, seed=3)), cdf_bits=16)
    rng = np.random.default_rng(7)
    batches = [[rng.integers(0, 300, n).astype(np.int32) for n in lens]
               for lens in ((5, 90, 33), (1,), (200, 200), (64, 3, 17, 120))]
    want = [codec.compress_tokens(b) for b in batches]
    assert list(codec.compress_batches(batches)) == want
    assert list(codec.compress_batches([])) == []


def _oracle_size(w, seqs, bits, key):
    """Bytes of the CPU oracle pipeline: fp32 forward (oracle/rwkv.py, pinned
    to rwkv4_step_ref) -> CDF rule of krunch_ac/cdf.py:22-74 -> range coder
    of krunch_ac/cpu_reference.py:91-147."""
    from oracle import coder, rwkv
    total = 0
    for i, s in enumerate(seqs):
        if (key, i) not in _ORACLE_LOGITS:
            inp = np.concatenate([[0], s[:-1]])[None]
            _ORACLE_LOGITS[key, i] = rwkv.forward(w, inp)[0][0].astype(np.float16)
        lh = coder.lohi_from_logits(_ORACLE_LOGITS[key, i], s, bits)
        total += len(coder.encode_lohi(lh, bits))
    return total


def _gpu_size(w, seqs, bits, wdtype="f16"):
    from krunch_b200.codec import Codec
    from krunch_b200.model import RWKVModel
    codec = Codec(RWKVModel(w, wdtype=wdtype), cdf_bits=bits)
    streams = codec.compress_tokens(seqs)
    back = codec.decompress_tokens(streams, [len(s) for s in seqs])
    for a, b in zip(seqs, back):
        assert np.array_equal(a, b)
    return sum(map(len, streams))


@pytest.mark.parametrize("bits", [16, 24])
def test_size_within_half_percent_of_oracle_169m(torch, bits):
    """BASELINE: compressed size within 0.5 % of the reference pipeline, on
    a model whose counts carry information."""
    w, seqs = _peaked()
    ours, ref = _gpu_size(w, seqs, bits), _oracle_size(w, seqs, bits, "f32")
    assert ref * 8 / sum(map(len, seqs)) < 8.0, "model not peaked: the test would have no teeth"
    assert abs(ours - ref) <= 0.005 * ref, (ours, ref)


def test_size_test_has_teeth(torch):
    """The same bar fails for a wrong model: one layer's attention output
    matrix zeroed (on the CPU oracle this costs 12-18 % more bytes)."""
    w, seqs = _peaked()
    bad = dict(w)
    bad["blocks.5.att.output.weight"] = np.zeros_like(w["blocks.5.att.output.weight"])
    ours, ref = _gpu_size(bad, seqs, 16), _oracle_size(w, seqs, 16, "f32")
    assert ours > 1.005 * ref, (ours, ref)


@pytest.mark.parametrize("bits", [16, 24])
def test_w8a8_size_vs_fp32_oracle(torch, bits):
    """The w8a8 model (the decompress model) has no
    reference kernel; its ratio cost is measured against the fp32 oracle
    pipeline: within 0.5 %."""
    w, seqs = _peaked()
    ours, ref = _gpu_size(w, seqs, bits, wdtype="i8"), _oracle_size(w, seqs, bits, "f32")
    assert abs(ours - ref) <= 0.005 * ref, (ours, ref)


@pytest.fixture()
def tiny_env(monkeypatch):
    monkeypatch.setenv("KRUNCH_MODEL", "tiny")
    monkeypatch.setenv("KRUNCH_TOKENIZER", "byte")
    monkeypatch.setenv("KRUNCH_CDF_BITS", "16")


def test_engine_chunks_roundtrip(torch, tiny_env):
    from krunch_b200.inference import InferenceEngine
    e = InferenceEngine()
    e.load()
    chunks = [markov_text(3000, seed=2), b"x", "héllo wörld ✓ ".encode() * 40, bytes(range(256))]
    enc = e.compress_chunks_batched(chunks)
    assert e.decompress_chunks_batched(enc) == chunks
    assert e.decompress_chunk(e.compress_chunk(chunks[0])) == chunks[0]


def test_cli_roundtrip_and_corruption(torch, tiny_env, tmp_path):
    raw = markov_text(20_000, seed=3)
    src, blob, back = tmp_path / "in", tmp_path / "blob", tmp_path / "out"
    src.write_bytes(raw)
    env = dict(os.environ, KRUNCH_CHUNK_SIZE="4096", PYTHONPATH=REPO)
    run = lambda *a: subprocess.run([sys.executable, "-m", "krunch_b200.cli", *a], env=env,  # noqa
                                    capture_output=True, timeout=600)
    r = run("compress", "--in", str(src), "--out", str(blob))
    assert r.returncode == 0, r.stderr.decode()[-2000:]
    r = run("decompress", "--in", str(blob), "--out", str(back))
    assert r.returncode == 0, r.stderr.decode()[-2000:]
    assert back.read_bytes() == raw
    data = bytearray(blob.read_bytes())
    data[-3] ^= 0x40  # corrupt the last chunk's bitstream -> CRC mismatch
    bad = tmp_path / "bad"
    bad.write_bytes(bytes(data))
    r = run("decompress", "--in", str(bad), "--out", str(tmp_path / "x"))
    assert r.returncode != 0


@pytest.mark.parametrize("raw", [b"", b"\x00", b"a", "\u20ac".encode()])
def test_cli_tiny_inputs(torch, tiny_env, tmp_path, raw):
    """Empty and one-byte inputs through the CLI (0 chunks / 1 chunk of one
    token): the blob round-trips, length and CRC checked on the way back."""
    src, blob, back = tmp_path / "in", tmp_path / "blob", tmp_path / "out"
    src.write_bytes(raw)
    env = dict(os.environ, PYTHONPATH=REPO)
    run = lambda *a: subprocess.run([sys.executable, "-m", "krunch_b200.cli", *a], env=env,  # noqa
                                    capture_output=True, timeout=600)
    r = run("compress", "--in", str(src), "--out", str(blob))
    assert r.returncode == 0, r.stderr.decode()[-2000:]
    r = run("decompress", "--in", str(blob), "--out", str(back))
    assert r.returncode == 0, r.stderr.decode()[-2000:]
    assert back.read_bytes() == raw
