"""Chunking and entry framing with the reference's semantics (krunch/chunking.py).

* ``compute_chunk_size`` (chunking.py:42-62): max(64 KiB, ceil(total / (4 *
  target_B))), target_B = $KRUNCH_TARGET_B or 128, pinned by $KRUNCH_CHUNK_SIZE.
* ``_split_utf8_safe`` (115-138): chunk ends walk back off UTF-8 continuation
  bytes so no code point is split.
* entries are ``>II(orig_len, comp_len)`` + payload (141-148, 166-170).

Unlike the reference, compress always hands every chunk to the batched codec
at once: chunks are encoded together (B streams in one packed forward)
because a chunk's bits do not depend on which other chunks share its batch.
"""
from __future__ import annotations

import logging
import os
import struct
from typing import Callable, Optional

logger = logging.getLogger(__name__)

_CHUNK_SIZE_FLOOR = 64 * 1024
_DEFAULT_TARGET_B = 128
CHUNK_SIZE = int(os.environ.get("KRUNCH_CHUNK_SIZE", _CHUNK_SIZE_FLOOR))
ENTRY_FMT = ">II"
ENTRY_SIZE = struct.calcsize(ENTRY_FMT)


def compute_chunk_size(total_size: int) -> int:
    explicit = os.environ.get("KRUNCH_CHUNK_SIZE")
    if explicit is not None:
        return int(explicit)
    if total_size <= 0:
        return _CHUNK_SIZE_FLOOR
    target_B = int(os.environ.get("KRUNCH_TARGET_B", _DEFAULT_TARGET_B))
    target_chunks = max(target_B * 4, 16)
    natural = (total_size + target_chunks - 1) // target_chunks
    return max(_CHUNK_SIZE_FLOOR, natural)


def _split_utf8_safe(raw: bytes, target_size: int) -> list[bytes]:
    if target_size <= 0:
        raise ValueError("chunk size must be positive")
    chunks = []
    pos, n = 0, len(raw)
    while pos < n:
        end = min(pos + target_size, n)
        if end < n:
            while end > pos and 0x80 <= raw[end] < 0xC0:
                end -= 1
            if end == pos:  # a run of continuation bytes longer than the chunk
                end = min(pos + target_size, n)
        chunks.append(raw[pos:end])
        pos = end
    return chunks


def split(raw: bytes, chunk_size: Optional[int] = None,
          total_size: Optional[int] = None) -> list[bytes]:
    if chunk_size is None:
        chunk_size = compute_chunk_size(total_size if total_size is not None else len(raw))
    return _split_utf8_safe(raw, chunk_size)


def pack_entries(chunks: list[bytes], payloads: list[bytes]) -> list[bytes]:
    return [struct.pack(ENTRY_FMT, len(c), len(z)) + z for c, z in zip(chunks, payloads)]


def compress_all(raw: bytes, neural_fn: Callable[[bytes], bytes],
                 neural_batch_fn: Optional[Callable[[list], list]] = None,
                 chunk_size: Optional[int] = None, total_size: Optional[int] = None,
                 ) -> tuple[list[bytes], int]:
    chunks = split(raw, chunk_size, total_size)
    if neural_batch_fn is not None and len(chunks) > 1:
        payloads = neural_batch_fn(chunks)
    else:
        payloads = [neural_fn(c) for c in chunks]
    entries = pack_entries(chunks, payloads)
    return entries, len(entries)


def parse_entries(entries_bytes: bytes, n_chunks: int) -> list[tuple[int, bytes]]:
    """[(orig_len, payload)] with bounds checks on every entry."""
    pos, out = 0, []
    for i in range(n_chunks):
        if pos + ENTRY_SIZE > len(entries_bytes):
            raise ValueError(f"truncated blob: entry {i} header missing")
        orig_len, comp_len = struct.unpack(ENTRY_FMT, entries_bytes[pos:pos + ENTRY_SIZE])
        pos += ENTRY_SIZE
        if pos + comp_len > len(entries_bytes):
            raise ValueError(f"truncated blob: entry {i} payload cut short")
        out.append((orig_len, entries_bytes[pos:pos + comp_len]))
        pos += comp_len
    return out


def decompress_all(entries_bytes: bytes, n_chunks: int, neural_fn: Callable[[bytes], bytes],
                   neural_batch_fn: Optional[Callable[[list], list]] = None) -> bytes:
    chunks = parse_entries(entries_bytes, n_chunks)
    if neural_batch_fn is not None and len(chunks) > 1:
        decoded = neural_batch_fn([enc for _, enc in chunks])
        return b"".join(d[:ol] for (ol, _), d in zip(chunks, decoded))
    return b"".join(neural_fn(enc)[:ol] for ol, enc in chunks)
