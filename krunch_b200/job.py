"""Multi-part compress / decompress jobs over local files: the worker and
finalize modes of the reference's batch job (krunch/job.py:55-256), driven
by the same environment variables, with local paths (or file:// URLs) in
place of the reference's object-store I/O (krunch/url_io.py, out of scope).

* compress worker  KRUNCH_MODE=compress: bytes [start, end) of the input
  (``byte_range``: equal chunk-aligned shares, job.py:243-256) become a part
  blob ``<output>.parts/part-NNNNNN`` whose header carries the part's own
  length and CRC32.  Chunk boundaries are those of a single-process compress
  of the whole input (every worker derives the chunk size from the total).
* decompress worker  KRUNCH_MODE=decompress: chunks [lo, hi) of the blob,
  ceil(n_chunks / part_count) per part (job.py:147-160), to raw bytes.
* finalize  KRUNCH_MODE=finalize, KRUNCH_FINALIZE_OF=compress|decompress:
  concatenates the parts in index order and removes them.  Unlike the
  reference, which writes crc 0 with the no-CRC flag (job.py:206), the
  compress finalize combines the parts' CRC32s into the CRC32 of the whole
  input (``crc32_combine``), so the master blob is fully verified on
  decompress.  It is byte-identical to a single-process compress whenever no
  part boundary falls inside a UTF-8 sequence (a single process would move
  such a chunk boundary back to the sequence start; a part boundary is hard).
  The decompress finalize checks length and CRC32 against the source blob's
  header when KRUNCH_INPUT_URL names it.
"""
from __future__ import annotations

import logging
import os
import sys
import zlib
from pathlib import Path
from typing import Callable

from . import chunking
from .inference import FLAG_NO_CRC, HEADER_SIZE, decode_header, encode_header

logger = logging.getLogger(__name__)


# ---- CRC32 of a concatenation (zlib's crc32_combine, restated) -------------
# The CRC register advances over len2 zero bytes by repeated squaring of the
# 32x32 GF(2) matrix of one zero bit; crc(A + B) = shift(crc(A), len(B)) ^
# crc(B) for the reflected polynomial 0xEDB88320.

def _gf2_times(mat: list[int], vec: int) -> int:
    out, i = 0, 0
    while vec:
        if vec & 1:
            out ^= mat[i]
        vec >>= 1
        i += 1
    return out


def _gf2_square(mat: list[int]) -> list[int]:
    return [_gf2_times(mat, mat[n]) for n in range(32)]


def crc32_combine(crc1: int, crc2: int, len2: int) -> int:
    """CRC32 of A + B from crc1 = CRC32(A), crc2 = CRC32(B), len2 = len(B)."""
    if len2 <= 0:
        return crc1 & 0xFFFFFFFF
    odd = [0xEDB88320] + [1 << n for n in range(31)]  # one zero bit
    even = _gf2_square(odd)                              # two zero bits
    odd = _gf2_square(even)                              # four zero bits
    crc1 &= 0xFFFFFFFF
    while True:  # apply len2 zero bytes: square through the bits of len2
        even = _gf2_square(odd)
        if len2 & 1:
            crc1 = _gf2_times(even, crc1)
        len2 >>= 1
        if not len2:
            break
        odd = _gf2_square(even)
        if len2 & 1:
            crc1 = _gf2_times(odd, crc1)
        len2 >>= 1
        if not len2:
            break
    return (crc1 ^ crc2) & 0xFFFFFFFF


# ---- byte and chunk ranges --------------------------------------------------

def byte_range(part_index: int, part_count: int, total_size: int) -> tuple[int, int]:
    """[start, end) of a compress part: equal shares rounded down to the
    chunk size every worker derives from total_size (job.py:243-256)."""
    chunk = chunking.compute_chunk_size(total_size)
    per_part = max((total_size // part_count // chunk) * chunk, chunk)
    start = part_index * per_part
    end = start + per_part if part_index < part_count - 1 else total_size
    return min(start, total_size), min(end, total_size)


def chunk_range(part_index: int, part_count: int, n_chunks: int) -> tuple[int, int]:
    """[lo, hi) chunk indices of a decompress part (job.py:147-160)."""
    per = (n_chunks + part_count - 1) // part_count
    lo = min(part_index * per, n_chunks)
    return lo, min(lo + per, n_chunks)


# ---- parts ------------------------------------------------------------------

def compress_part(raw_part: bytes, total_size: int,
                  compress_batch: Callable[[list], list]) -> bytes:
    """Part blob of one byte range: header (part length, chunk count, part
    CRC32) + entries, chunked as the whole input would be."""
    chunks = chunking.split(raw_part, total_size=total_size)
    payloads = compress_batch(chunks) if chunks else []
    crc = zlib.crc32(raw_part) & 0xFFFFFFFF
    return encode_header(len(raw_part), len(chunks), crc) + b"".join(
        chunking.pack_entries(chunks, payloads))


def finalize_compress(parts: list[bytes], original_len: int) -> bytes:
    """Master blob of the parts in index order, with the CRC32 of the whole
    input combined from the parts' CRC32s (flags 0)."""
    crc, total, n_chunks, entries = 0, 0, 0, []
    for i, blob in enumerate(parts):
        hdr = decode_header(blob)
        if hdr["flags"] & FLAG_NO_CRC:
            raise ValueError(f"part {i} carries no CRC32")
        crc = crc32_combine(crc, hdr["crc32"], hdr["original_len"]) if i else hdr["crc32"]
        total += hdr["original_len"]
        n_chunks += hdr["n_chunks"]
        entries.append(blob[HEADER_SIZE:])
    if total != original_len:
        raise ValueError(f"parts hold {total} bytes, the input has {original_len}")
    first = decode_header(parts[0]) if parts else None
    return encode_header(original_len, n_chunks, crc,
                         model_id=None if first is None else first["model_id"],
                         tokenizer_id=None if first is None else first["tokenizer_id"]
                         ) + b"".join(entries)


def decompress_part(blob: bytes, part_index: int, part_count: int,
                    decompress_batch: Callable[[list], list]) -> bytes:
    """Raw bytes of this part's chunk range of a blob."""
    hdr = decode_header(blob)
    entries = chunking.parse_entries(blob[HEADER_SIZE:], hdr["n_chunks"])
    lo, hi = chunk_range(part_index, part_count, len(entries))
    mine = entries[lo:hi]
    if not mine:
        return b""
    decoded = decompress_batch([enc for _, enc in mine])
    return b"".join(d[:ol] for (ol, _), d in zip(mine, decoded))


def check_raw(raw: bytes, hdr: dict) -> None:
    """Length and (unless the blob carries none) CRC32 of a reassembled
    output against the source blob's header; ValueError on a mismatch."""
    if len(raw) != hdr["original_len"]:
        raise ValueError(f"length mismatch: got {len(raw)}, expected {hdr['original_len']}")
    if not hdr["flags"] & FLAG_NO_CRC:
        actual = zlib.crc32(raw) & 0xFFFFFFFF
        if actual != hdr["crc32"]:
            raise ValueError(f"CRC32 mismatch: got {actual:#010x}, expected {hdr['crc32']:#010x}")


# ---- the job entry point (local files) ----------------------------------------

def _path(url: str) -> Path:
    if url.startswith("file://"):
        return Path(url[len("file://"):])
    if "://" in url:
        raise ValueError(f"only local paths and file:// URLs are supported, got {url!r}")
    return Path(url)


def parts_dir(output_url: str) -> Path:
    """Parts live beside the final output (job.py:238-240)."""
    return Path(str(_path(output_url)).rstrip("/") + ".parts")


def part_path(output_url: str, i: int) -> Path:
    return parts_dir(output_url) / f"part-{i:06d}"


def run(env=None) -> None:
    env = os.environ if env is None else env
    mode = env.get("KRUNCH_MODE", "").lower()
    out = env["KRUNCH_OUTPUT_URL"]
    count = int(env["KRUNCH_PART_COUNT"])
    if mode in ("compress", "decompress"):
        from .inference import engine
        idx = int(env["KRUNCH_PART_INDEX"])
        engine.load()
        src = _path(env["KRUNCH_INPUT_URL"])
        if mode == "compress":
            total = int(env["KRUNCH_INPUT_LEN"])
            start, end = byte_range(idx, count, total)
            with open(src, "rb") as f:
                f.seek(start)
                raw = f.read(end - start)
            data = compress_part(raw, total, engine.compress_chunks_batched)
        else:
            blob = src.read_bytes()
            engine.configure_from_header(decode_header(blob))
            data = decompress_part(blob, idx, count, engine.decompress_chunks_batched)
        p = part_path(out, idx)
        p.parent.mkdir(parents=True, exist_ok=True)
        p.write_bytes(data)
        logger.info("%s part %d/%d: %d bytes -> %s", mode, idx, count, len(data), p)
    elif mode == "finalize":
        parts = [part_path(out, i).read_bytes() for i in range(count)]
        if env.get("KRUNCH_FINALIZE_OF", "compress").lower() == "compress":
            data = finalize_compress(parts, int(env["KRUNCH_INPUT_LEN"]))
        else:
            data = b"".join(parts)
            if env.get("KRUNCH_INPUT_URL"):
                with open(_path(env["KRUNCH_INPUT_URL"]), "rb") as f:
                    check_raw(data, decode_header(f.read(HEADER_SIZE)))
        _path(out).write_bytes(data)
        for i in range(count):
            part_path(out, i).unlink(missing_ok=True)
        logger.info("finalize: %d bytes -> %s", len(data), out)
    else:
        logger.error("KRUNCH_MODE must be 'compress'|'decompress'|'finalize', got %r", mode)
        sys.exit(1)


if __name__ == "__main__":
    logging.basicConfig(level=logging.INFO)
    run()
