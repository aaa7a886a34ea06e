"""``krunch compress|decompress [--in PATH] [--out PATH]`` (krunch/cli.py:137-154).

stdin/stdout by default; stdout carries only the blob (logs go to stderr).
Compress writes header + entries with CRC32 over the raw input (flags 0);
decompress checks the CRC (unless flags & 1) and the length, exiting non-zero
on a mismatch (cli.py:106-116).  With torchrun (WORLD_SIZE > 1) the chunks are
sharded round-robin over the ranks and rank 0 writes the stitched blob, which
is byte-identical to the single-GPU one.
"""
from __future__ import annotations

import argparse
import contextlib
import logging
import os
import sys
import zlib

from . import chunking
from .inference import HEADER_SIZE, FLAG_NO_CRC, decode_header, encode_header, engine

logging.basicConfig(level=logging.INFO, format="%(asctime)s %(levelname)s %(message)s",
                    stream=sys.stderr)
logger = logging.getLogger("krunch_b200.cli")


@contextlib.contextmanager
def _stdout_to_stderr():
    """FD 1 -> FD 2 while loading, so nothing but the blob reaches stdout."""
    saved = os.dup(1)
    try:
        os.dup2(2, 1)
        yield
    finally:
        os.dup2(saved, 1)
        os.close(saved)


def _read_input(path):
    if path and path != "-":
        with open(path, "rb") as f:
            return f.read()
    return sys.stdin.buffer.read()


def _write_output(path, data: bytes) -> None:
    if path and path != "-":
        with open(path, "wb") as f:
            f.write(data)
    else:
        sys.stdout.buffer.write(data)
        sys.stdout.buffer.flush()


def compress_bytes(raw: bytes) -> bytes:
    from . import distributed as dist
    chunks = chunking.split(raw)
    payloads = dist.map_chunks(engine.compress_chunks_batched, chunks)
    if payloads is None:  # non-zero rank
        return b""
    crc = zlib.crc32(raw) & 0xFFFFFFFF
    return encode_header(len(raw), len(chunks), crc) + b"".join(
        chunking.pack_entries(chunks, payloads))


def decompress_bytes(blob: bytes) -> bytes:
    from . import distributed as dist
    hdr = decode_header(blob)
    with _stdout_to_stderr():
        engine.configure_from_header(hdr)
    entries = chunking.parse_entries(blob[HEADER_SIZE:], hdr["n_chunks"])
    decoded = dist.map_chunks(engine.decompress_chunks_batched, [enc for _, enc in entries])
    if decoded is None:
        return b""
    raw = b"".join(d[:ol] for (ol, _), d in zip(entries, decoded))
    if not hdr["flags"] & FLAG_NO_CRC:
        actual = zlib.crc32(raw) & 0xFFFFFFFF
        if actual != hdr["crc32"]:
            raise SystemExit(f"CRC32 mismatch: got {actual:#010x}, expected {hdr['crc32']:#010x}")
    if len(raw) != hdr["original_len"]:
        raise SystemExit(f"length mismatch: got {len(raw)}, expected {hdr['original_len']}")
    return raw


def cmd_compress(args) -> None:
    from . import distributed as dist
    raw = _read_input(args.input)
    with _stdout_to_stderr():
        engine.load(device=dist.local_device())
    blob = compress_bytes(raw)
    if dist.rank() == 0:
        _write_output(args.output, blob)
        logger.info("compress %d -> %d bytes (%.4f)", len(raw), len(blob),
                    len(blob) / len(raw) if raw else 0.0)


def cmd_decompress(args) -> None:
    from . import distributed as dist
    blob = _read_input(args.input)
    with _stdout_to_stderr():
        engine.load(device=dist.local_device())
    raw = decompress_bytes(blob)
    if dist.rank() == 0:
        _write_output(args.output, raw)
        logger.info("decompress %d -> %d bytes", len(blob), len(raw))


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(prog="krunch", description="Krunch neural compression (B200)")
    sub = ap.add_subparsers(dest="cmd", required=True)
    for name, hlp in (("compress", "Compress bytes"), ("decompress", "Decompress a .krunch blob")):
        p = sub.add_parser(name, help=hlp)
        p.add_argument("--in", dest="input", help="Input file (default: stdin)")
        p.add_argument("--out", dest="output", help="Output file (default: stdout)")
    args = ap.parse_args(argv)
    from . import distributed as dist
    dist.init_from_env()
    try:
        (cmd_compress if args.cmd == "compress" else cmd_decompress)(args)
    finally:
        dist.shutdown()


if __name__ == "__main__":
    main()
