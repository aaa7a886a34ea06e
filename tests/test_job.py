"""Multi-part job workers and finalize (reference krunch/job.py:55-256),
host only: the neural coder is replaced by a stand-in so the chunk
framing, byte/chunk ranges and CRC combination are what is tested."""
import os
import random
import zlib

import pytest

from krunch_b200 import chunking, inference, job
from krunch_b200.inference import HEADER_SIZE, decode_header, encode_header


def _fake_c(chunks):
    return [zlib.compress(c, 1) for c in chunks]


def _fake_d(encs):
    return [zlib.decompress(e) for e in encs]


def _single(raw):
    chunks = chunking.split(raw)
    crc = zlib.crc32(raw) & 0xFFFFFFFF
    return encode_header(len(raw), len(chunks), crc) + b"".join(
        chunking.pack_entries(chunks, _fake_c(chunks)))


def test_crc32_combine_matches_zlib():
    rng = random.Random(7)
    for _ in range(40):
        a = rng.randbytes(rng.randrange(0, 3000))
        b = rng.randbytes(rng.randrange(0, 3000))
        assert job.crc32_combine(zlib.crc32(a), zlib.crc32(b), len(b)) == zlib.crc32(a + b)
    big = bytes(range(256)) * 4099
    assert job.crc32_combine(zlib.crc32(b"x"), zlib.crc32(big), len(big)) == zlib.crc32(b"x" + big)


@pytest.mark.parametrize("total,parts", [(0, 3), (10, 4), (5000, 1), (70000, 3), (70001, 7), (1 << 20, 8)])
def test_byte_range_tiles_input(total, parts):
    ranges = [job.byte_range(i, parts, total) for i in range(parts)]
    assert ranges[0][0] == 0 and ranges[-1][1] == total
    chunk = chunking.compute_chunk_size(total)
    for (s0, e0), (s1, e1) in zip(ranges, ranges[1:]):
        assert e0 == s1 and s0 <= e0
    for s, e in ranges[:-1]:
        assert s % chunk == 0 or s == total
        assert e % chunk == 0 or e == total


@pytest.mark.parametrize("n,parts", [(0, 2), (1, 4), (7, 3), (16, 4), (17, 16)])
def test_chunk_range_tiles_entries(n, parts):
    rs = [job.chunk_range(i, parts, n) for i in range(parts)]
    assert rs[0][0] == 0 and rs[-1][1] == n
    assert all(a[1] == b[0] for a, b in zip(rs, rs[1:]))


@pytest.mark.parametrize("parts", [1, 2, 3, 5])
def test_finalize_equals_single_process(parts, monkeypatch):
    monkeypatch.setenv("KRUNCH_CHUNK_SIZE", "4096")
    raw = (b"the quick brown fox jumps over the lazy dog. " * 3000)[:123457]
    pblobs = []
    for i in range(parts):
        s, e = job.byte_range(i, parts, len(raw))
        pblobs.append(job.compress_part(raw[s:e], len(raw), _fake_c))
        assert decode_header(pblobs[-1])["crc32"] == zlib.crc32(raw[s:e])
    master = job.finalize_compress(pblobs, len(raw))
    assert master == _single(raw)
    hdr = decode_header(master)
    assert hdr["flags"] == 0 and hdr["crc32"] == zlib.crc32(raw)
    out = b"".join(job.decompress_part(master, i, 4, _fake_d) for i in range(4))
    assert out == raw
    job.check_raw(out, hdr)
    with pytest.raises(ValueError):
        job.check_raw(out[:-1] + b"X", hdr)


def test_finalize_rejects_missing_bytes_and_crcless_parts():
    a = job.compress_part(b"abc" * 100, 600, _fake_c)
    with pytest.raises(ValueError):
        job.finalize_compress([a], 600)
    nocrc = encode_header(3, 1, 0, flags=inference.FLAG_NO_CRC) + a[HEADER_SIZE:]
    with pytest.raises(ValueError):
        job.finalize_compress([nocrc], 3)


class _FakeEngine:
    model_id = tokenizer_id = 1

    def load(self, *a, **k):
        pass

    def configure_from_header(self, hdr):
        self.hdr = hdr

    compress_chunks_batched = staticmethod(_fake_c)
    decompress_chunks_batched = staticmethod(_fake_d)


def test_run_env_driven_job(tmp_path, monkeypatch):
    monkeypatch.setenv("KRUNCH_CHUNK_SIZE", "1000")
    monkeypatch.setattr(inference, "engine", _FakeEngine())
    raw = os.urandom(2000) + "héllo wörld ".encode() * 700
    src = tmp_path / "in.bin"
    src.write_bytes(raw)
    blob = tmp_path / "out.krunch"
    base = {"KRUNCH_INPUT_URL": str(src), "KRUNCH_OUTPUT_URL": "file://" + str(blob),
            "KRUNCH_PART_COUNT": "3", "KRUNCH_INPUT_LEN": str(len(raw))}
    for i in range(3):
        job.run({**base, "KRUNCH_MODE": "compress", "KRUNCH_PART_INDEX": str(i)})
    job.run({**base, "KRUNCH_MODE": "finalize", "KRUNCH_FINALIZE_OF": "compress"})
    assert not list(job.parts_dir(str(blob)).iterdir())
    assert decode_header(blob.read_bytes())["crc32"] == zlib.crc32(raw)
    out = tmp_path / "back.bin"
    dbase = {"KRUNCH_INPUT_URL": str(blob), "KRUNCH_OUTPUT_URL": str(out), "KRUNCH_PART_COUNT": "2"}
    for i in range(2):
        job.run({**dbase, "KRUNCH_MODE": "decompress", "KRUNCH_PART_INDEX": str(i)})
    job.run({**dbase, "KRUNCH_MODE": "finalize", "KRUNCH_FINALIZE_OF": "decompress"})
    assert out.read_bytes() == raw
    with pytest.raises(SystemExit):
        job.run({**dbase, "KRUNCH_MODE": "bogus"})
