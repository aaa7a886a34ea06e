"""Blob header, entry framing and chunking (reference tests/test_blob.py,
tests/test_utf8_chunking.py), host only."""
import struct
import zlib

import pytest

from krunch_b200 import chunking
from krunch_b200.chunking import (_CHUNK_SIZE_FLOOR, _split_utf8_safe, compress_all,
                                  compute_chunk_size, decompress_all, parse_entries)
from krunch_b200.inference import (BLOB_MAGIC, HEADER_SIZE, CodecConfig, decode_header,
                                   encode_header)


def test_header_roundtrip_and_size():
    assert HEADER_SIZE == 37 == struct.calcsize(">4sBIIIHHQII")
    h = encode_header(123456, 7, 0xDEADBEEF, model_id=1, tokenizer_id=1)
    assert len(h) == HEADER_SIZE and h[:4] == BLOB_MAGIC
    p = decode_header(h)
    assert (p["original_len"], p["n_chunks"], p["crc32"], p["blob_version"], p["model_id"]) == \
        (123456, 7, 0xDEADBEEF, 1, 1)
    with pytest.raises(ValueError):
        decode_header(b"XXXX" + h[4:])
    with pytest.raises(ValueError):
        decode_header(h[:10])


def test_model_id_roundtrip():
    for cfg in (CodecConfig(), CodecConfig("tiny", 3, 16, "production", "f16")):
        assert CodecConfig.from_model_id(cfg.model_id) == cfg
    with pytest.raises(RuntimeError):
        CodecConfig.from_model_id(1)  # the reference's pretrained-weights id


def test_compute_chunk_size(monkeypatch):
    monkeypatch.delenv("KRUNCH_CHUNK_SIZE", raising=False)
    monkeypatch.delenv("KRUNCH_TARGET_B", raising=False)
    assert compute_chunk_size(10_000) == _CHUNK_SIZE_FLOOR
    assert compute_chunk_size(0) == _CHUNK_SIZE_FLOOR
    assert compute_chunk_size(10 * 1024 * 1024) == _CHUNK_SIZE_FLOOR
    assert compute_chunk_size(100 * 1024 * 1024) == 200 * 1024
    assert compute_chunk_size(1024 * 1024 * 1024) == 2 * 1024 * 1024
    monkeypatch.setenv("KRUNCH_TARGET_B", "512")
    assert compute_chunk_size(1024 * 1024 * 1024) == 512 * 1024
    monkeypatch.setenv("KRUNCH_CHUNK_SIZE", "131072")
    assert compute_chunk_size(1000) == 131072


def test_utf8_split():
    raw = b"a" * 100_000
    ch = _split_utf8_safe(raw, 1024)
    assert b"".join(ch) == raw and all(len(c) == 1024 for c in ch[:-1])
    raw = (b"x" + b"\xe2\x80\x9c") * 10_000
    ch = _split_utf8_safe(raw, 1023)
    assert b"".join(ch) == raw
    for c in ch:
        c.decode("utf-8")
    raw = b"\xe2\x80\x9c" * 5
    ch = _split_utf8_safe(raw, 4)
    assert b"".join(ch) == raw and all(c.decode("utf-8") for c in ch)
    assert _split_utf8_safe(b"", 1024) == []
    assert _split_utf8_safe(b"hello world", 1024) == [b"hello world"]
    # invalid UTF-8 (a long run of continuation bytes) still splits losslessly
    raw = b"\x80" * 5000
    assert b"".join(_split_utf8_safe(raw, 1000)) == raw


def _xor(b):
    return bytes(x ^ 0x5A for x in b)


@pytest.mark.parametrize("batched", [False, True])
def test_chunking_roundtrip(batched):
    raw = b"Hello, Krunch! " * 20_000
    bf = (lambda cs: [_xor(c) for c in cs]) if batched else None
    entries, n = compress_all(raw, _xor, neural_batch_fn=bf, chunk_size=4096)
    assert n == len(entries) == (len(raw) + 4095) // 4096
    blob = b"".join(entries)
    assert decompress_all(blob, n, _xor, neural_batch_fn=bf) == raw
    entries2, n2 = compress_all(raw, _xor, total_size=10 * 1024 * 1024)
    assert decompress_all(b"".join(entries2), n2, _xor) == raw


def test_truncated_entries_raise():
    entries, n = compress_all(b"abc" * 50_000, _xor, chunk_size=10_000)
    blob = b"".join(entries)
    with pytest.raises(ValueError):
        parse_entries(blob[:-1], n)
    with pytest.raises(ValueError):
        parse_entries(blob[:5], n)
    assert len(parse_entries(blob, n)) == n


def test_crc_detects_corruption():
    data = b"test data for crc" * 100
    bad = bytearray(data)
    bad[50] ^= 0xFF
    assert zlib.crc32(bytes(bad)) != zlib.crc32(data)
