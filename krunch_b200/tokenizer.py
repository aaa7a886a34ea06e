"""Tokenisers behind the codec (the reference's step: krunch/inference.py:225-226
encode, 441-442 decode).

* ``NeoXTokenizer`` (tokenizer_id 1) — the reference's GPT-NeoX BPE, used when
  ``$KRUNCH_MODEL_DIR/20B_tokenizer.json`` exists.  Like the reference it
  tokenises ``data.decode("utf-8", errors="replace")``, so it is lossless only
  for valid UTF-8 input.
* ``ByteTokenizer`` (tokenizer_id 2) — one token per byte (id = byte value).
  Lossless for any input; the default when no tokenizer file is supplied.
"""
from __future__ import annotations

import os
from pathlib import Path

import numpy as np


class ByteTokenizer:
    tokenizer_id = 2
    name = "byte"

    def encode(self, data: bytes) -> np.ndarray:
        return np.frombuffer(bytes(data), dtype=np.uint8).astype(np.int32)

    def decode(self, ids) -> bytes:
        a = np.asarray(ids, dtype=np.int64)
        if a.size and (a.min() < 0 or a.max() > 255):
            raise ValueError("byte tokenizer: id outside [0, 255]")
        return a.astype(np.uint8).tobytes()


class NeoXTokenizer:
    tokenizer_id = 1
    name = "neox"

    def __init__(self, path: Path):
        from tokenizers import Tokenizer
        self._tok = Tokenizer.from_file(str(path))

    def encode(self, data: bytes) -> np.ndarray:
        text = bytes(data).decode("utf-8", errors="replace")
        return np.asarray(self._tok.encode(text).ids, dtype=np.int32)

    def decode(self, ids) -> bytes:
        return self._tok.decode([int(i) for i in ids]).encode("utf-8")


def model_dir() -> Path:
    return Path(os.environ.get("KRUNCH_MODEL_DIR", "/models"))


def load_tokenizer(kind: str | None = None):
    kind = kind or os.environ.get("KRUNCH_TOKENIZER", "auto")
    path = model_dir() / "20B_tokenizer.json"
    if kind == "neox" or (kind == "auto" and path.exists()):
        return NeoXTokenizer(path)
    if kind in ("byte", "auto"):
        return ByteTokenizer()
    raise ValueError(f"unknown tokenizer {kind!r}")


def tokenizer_for_id(tid: int):
    if tid == ByteTokenizer.tokenizer_id:
        return ByteTokenizer()
    if tid == NeoXTokenizer.tokenizer_id:
        path = model_dir() / "20B_tokenizer.json"
        if not path.exists():
            raise RuntimeError(f"blob needs the GPT-NeoX tokenizer but {path} is missing")
        return NeoXTokenizer(path)
    raise ValueError(f"unknown tokenizer_id {tid}")
