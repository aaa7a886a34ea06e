"""End-to-end byte-exact round trips through the codec, the engine and the
CLI, and compressed size against the CPU oracle pipeline (BASELINE: within
0.5%)."""
import os
import subprocess
import sys

import numpy as np
import pytest

from krunch_b200.synth import markov_text, random_weights, zipf_tokens

pytestmark = pytest.mark.gpu
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


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


def _oracle_size(w, seqs, bits):
    from oracle import coder, rwkv
    total = 0
    for s in seqs:
        inp = np.concatenate([[0], s[:-1]])[None]
        lg, _ = rwkv.forward(w, inp)
        lh = coder.lohi_from_logits(lg[0].astype(np.float16), s, bits)
        total += len(coder.encode_lohi(lh, bits))
    return total


@pytest.mark.parametrize("bits", [16, 24])
def test_size_within_half_percent_of_oracle_169m(torch, bits):
    from krunch_b200.codec import Codec
    from krunch_b200.model import RWKVModel
    w = random_weights(12, 768, 3072, 50277, seed=0)
    seqs = [zipf_tokens(n, seed=10 + n) for n in (400, 250)]
    codec = Codec(RWKVModel(w), cdf_bits=bits)
    streams = codec.compress_tokens(seqs)
    back = codec.decompress_tokens(streams, [len(s) for s in seqs])
    for a, b in zip(seqs, back):
        assert np.array_equal(a, b)
    ours, ref = sum(map(len, streams)), _oracle_size(w, seqs, bits)
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
