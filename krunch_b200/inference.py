"""Engine with the reference's krunch.inference surface (krunch/inference.py).

``engine`` (a module-level InferenceEngine) offers load / compress_chunk /
decompress_chunk / compress_chunks_batched / decompress_chunks_batched, and
the module keeps the .krunch header helpers (encode_header, decode_header,
HEADER_FMT, HEADER_SIZE = 37, BOS_TOKEN) byte-compatible with
inference.py:43-98.

Chunk payload (inference.py:289-291, 360): ``>II(orig_len, n_tokens)`` then
the range-coded bitstream.

What the engine runs is fixed by environment variables read at load():
  KRUNCH_MODEL        "169m" (default), "1b5" or "tiny" — random-init RWKV-4
                      (krunch_b200.synth.random_weights) of that shape;
  KRUNCH_WEIGHTS_SEED seed of those weights (default 0);
  KRUNCH_CDF_BITS     CDF total 2^bits (default 24, the reference's);
  KRUNCH_WKV          "step_ref" (default) or "production";
  KRUNCH_TOKENIZER    "auto" (default), "byte" or "neox".
Everything that changes bits is written into the blob header's model_id and
tokenizer_id, and decompress reconfigures itself from them, so a blob never
depends on the decoder's environment.
"""
from __future__ import annotations

import logging
import os
import struct
import time
from dataclasses import dataclass

import numpy as np

logger = logging.getLogger(__name__)

BLOB_MAGIC = b"KRNC"
BLOB_VERSION = 1
HEADER_FMT = ">4sBIIIHHQII"  # magic, version, model_id, tokenizer_id, adapter_id,
HEADER_SIZE = struct.calcsize(HEADER_FMT)  # adapter_version, flags, orig_len, n_chunks, crc32 = 37 B
BOS_TOKEN = 0
FLAG_NO_CRC = 0x01  # assembled-from-parts blobs (krunch/job.py:206, cli.py:106)

# model_id of the reference's real RWKV-4-Pile-169M weights (inference.py:50).
REFERENCE_MODEL_ID = 1
# "pile169m": the pretrained RWKV-4-Pile-169M checkpoint from $KRUNCH_MODEL_DIR
FAMILIES = {"169m": 1, "tiny": 2, "1b5": 3, "pile169m": 4}
SHAPES = {
    "169m": dict(n_layer=12, n_embd=768, n_ffn=3072, n_vocab=50277),
    "1b5": dict(n_layer=24, n_embd=2048, n_ffn=8192, n_vocab=50277),
    "tiny": dict(n_layer=2, n_embd=128, n_ffn=512, n_vocab=384),
    "pile169m": dict(n_layer=12, n_embd=768, n_ffn=3072, n_vocab=50277),
}
WDTYPES = {"f16": 0, "bf16": 1, "i8": 2}
WKVS = {"step_ref": 0, "production": 1}


@dataclass(frozen=True)
class CodecConfig:
    family: str = "169m"
    seed: int = 0
    cdf_bits: int = 24
    wkv: str = "step_ref"
    wdtype: str = "f16"

    @property
    def model_id(self) -> int:
        """u32: bits 0-7 cdf_bits, 8-11 weight dtype, 12-15 WKV convention,
        16-23 model family, 24-31 weight seed."""
        return (self.cdf_bits | WDTYPES[self.wdtype] << 8 | WKVS[self.wkv] << 12
                | FAMILIES[self.family] << 16 | (self.seed & 0xFF) << 24)

    @staticmethod
    def from_model_id(mid: int) -> "CodecConfig":
        if mid == REFERENCE_MODEL_ID:
            raise RuntimeError("blob was written by the reference with RWKV-4-Pile-169M "
                               "pretrained weights, which this installation does not have")
        inv = lambda d, v: {b: a for a, b in d.items()}[v]  # noqa: E731
        try:
            return CodecConfig(family=inv(FAMILIES, (mid >> 16) & 0xFF), seed=(mid >> 24) & 0xFF,
                               cdf_bits=mid & 0xFF, wkv=inv(WKVS, (mid >> 12) & 0xF),
                               wdtype=inv(WDTYPES, (mid >> 8) & 0xF))
        except KeyError:
            raise ValueError(f"unknown model_id {mid:#010x}") from None

    @staticmethod
    def from_env() -> "CodecConfig":
        return CodecConfig(family=os.environ.get("KRUNCH_MODEL", "169m"),
                           seed=int(os.environ.get("KRUNCH_WEIGHTS_SEED", "0")),
                           cdf_bits=int(os.environ.get("KRUNCH_CDF_BITS", "24")),
                           wkv=os.environ.get("KRUNCH_WKV", "step_ref"),
                           wdtype=os.environ.get("KRUNCH_WDTYPE", "f16"))


def encode_header(original_len: int, n_chunks: int, crc32: int, adapter_id: int = 0,
                  adapter_version: int = 0, flags: int = 0, model_id: int | None = None,
                  tokenizer_id: int | None = None) -> bytes:
    if model_id is None or tokenizer_id is None:
        model_id = engine.model_id if model_id is None else model_id
        tokenizer_id = engine.tokenizer_id if tokenizer_id is None else tokenizer_id
    return struct.pack(HEADER_FMT, BLOB_MAGIC, BLOB_VERSION, model_id, tokenizer_id, adapter_id,
                       adapter_version, flags, original_len, n_chunks, crc32)


def decode_header(data: bytes) -> dict:
    if len(data) < HEADER_SIZE:
        raise ValueError(f"blob too short: {len(data)} < {HEADER_SIZE}")
    magic, bv, mid, tid, aid, av, flags, orig_len, n_chunks, crc = struct.unpack(
        HEADER_FMT, data[:HEADER_SIZE])
    if magic != BLOB_MAGIC:
        raise ValueError(f"bad magic: {magic!r}")
    return {"blob_version": bv, "model_id": mid, "tokenizer_id": tid, "adapter_id": aid,
            "adapter_version": av, "flags": flags, "original_len": orig_len,
            "n_chunks": n_chunks, "crc32": crc}


_MODEL_CACHE: dict = {}


def build_model(cfg: CodecConfig, device="cuda"):
    """Device model for a config (cached per process and device)."""
    import torch
    from .model import RWKVModel
    from .synth import random_weights
    dev = torch.device(device)
    if dev.type == "cuda" and dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    key = (cfg.family, cfg.seed, cfg.wkv, cfg.wdtype, str(dev))
    if key not in _MODEL_CACHE:
        if cfg.family == "pile169m":
            from .weights import load_rwkv4_checkpoint, pretrained_path
            path = pretrained_path()
            if path is None:
                raise RuntimeError("pretrained RWKV-4-Pile-169M weights not found: set "
                                   "KRUNCH_MODEL_DIR to the directory holding them")
            w = load_rwkv4_checkpoint(path)
        else:
            w = random_weights(**SHAPES[cfg.family], seed=cfg.seed)
        _MODEL_CACHE[key] = RWKVModel(w, device=dev, wkv=cfg.wkv, wdtype=cfg.wdtype)
    return _MODEL_CACHE[key]


class InferenceEngine:
    def __init__(self):
        self._ready = False
        self.cfg: CodecConfig | None = None
        self._tok = None
        self._codec = None
        self.device = None

    # --------------------------------------------------------------- setup
    def load(self, cfg: CodecConfig | None = None, tokenizer=None, device=None):
        """Load model + tokenizer (GPU only; raises without CUDA)."""
        import torch
        from .codec import Codec
        from .tokenizer import load_tokenizer
        if not torch.cuda.is_available():
            raise RuntimeError("krunch_b200 needs a CUDA device")
        t0 = time.time()
        self.cfg = cfg or CodecConfig.from_env()
        self._tok = tokenizer or load_tokenizer()
        if self._tok.tokenizer_id == 2 and SHAPES[self.cfg.family]["n_vocab"] < 256:
            raise ValueError("byte tokenizer needs a vocabulary of at least 256")
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        model = build_model(self.cfg, self.device)
        self._codec = Codec(model, cdf_bits=self.cfg.cdf_bits)
        self._ready = True
        logger.info("krunch_b200 engine ready in %.1fs (%s, tokenizer=%s)", time.time() - t0,
                    self.cfg, self._tok.name)

    def configure_from_header(self, hdr: dict) -> None:
        """Make the engine match a blob's model_id / tokenizer_id."""
        from .tokenizer import tokenizer_for_id
        cfg = CodecConfig.from_model_id(hdr["model_id"])
        tok = self._tok if (self._tok is not None and
                            self._tok.tokenizer_id == hdr["tokenizer_id"]) \
            else tokenizer_for_id(hdr["tokenizer_id"])
        if not self._ready or cfg != self.cfg or tok is not self._tok:
            self.load(cfg, tok, self.device)

    @property
    def ready(self) -> bool:
        return self._ready

    @property
    def model_id(self) -> int:
        return (self.cfg or CodecConfig.from_env()).model_id

    @property
    def tokenizer_id(self) -> int:
        if self._tok is None:
            from .tokenizer import load_tokenizer
            return load_tokenizer().tokenizer_id
        return self._tok.tokenizer_id

    @property
    def codec(self):
        if not self._ready:
            self.load()
        return self._codec

    # ------------------------------------------------------------ chunks
    def _tokens(self, data: bytes) -> np.ndarray:
        toks = self._tok.encode(data)
        if len(toks) < 1:
            raise ValueError("chunk has no tokens after tokenization")
        return toks

    def compress_chunk(self, data: bytes) -> bytes:
        return self.compress_chunks_batched([data])[0]

    def compress_chunks_batched(self, chunks: list[bytes]) -> list[bytes]:
        if not chunks:
            return []
        codec = self.codec
        toks = [self._tokens(c) for c in chunks]
        streams = codec.compress_tokens(toks)
        return [struct.pack(">II", len(c), len(t)) + s for c, t, s in zip(chunks, toks, streams)]

    def decompress_chunk(self, encoded: bytes) -> bytes:
        return self.decompress_chunks_batched([encoded])[0]

    def decompress_chunks_batched(self, encoded_chunks: list[bytes]) -> list[bytes]:
        if not encoded_chunks:
            return []
        codec = self.codec
        orig, ntok, bss = [], [], []
        for enc in encoded_chunks:
            if len(enc) < 8:
                raise ValueError("truncated chunk: missing mini-header")
            ol, nt = struct.unpack(">II", enc[:8])
            orig.append(ol)
            ntok.append(nt)
            bss.append(enc[8:])
        toks = codec.decompress_tokens(bss, ntok)
        return [self._tok.decode(t)[:ol] for t, ol in zip(toks, orig)]


engine = InferenceEngine()
