"""numpy front end of oracle/kb_oracle.c — TEST INFRASTRUCTURE ONLY.

Range coder restated from krunch_ac/cpu_reference.py; CDF rule from
krunch_ac/cdf.py:22-74 evaluated in the GPU kernel's fixed order.
"""
from __future__ import annotations

import concurrent.futures as cf
import ctypes as C
import os

import numpy as np

from . import build as _build

_lib = None


def lib():
    global _lib
    if _lib is None:
        path = _build.build()
        L = C.CDLL(str(path))
        vp, i32, i64 = C.c_void_p, C.c_int, C.c_int64
        L.oc_expf.restype = C.c_float
        L.oc_expf.argtypes = [C.c_float]
        L.oc_cdf_from_logits.argtypes = [vp, i64, i32, i32, i32, vp]
        L.oc_cdf_from_probs.argtypes = [vp, i32, i32, i32, vp]
        L.oc_lohi_from_logits.argtypes = [vp, i64, i32, i32, i32, vp, vp]
        L.oc_encode_lohi.restype = i64
        L.oc_encode_lohi.argtypes = [vp, i64, i32, vp, i64]
        L.oc_encode_cdf.restype = i64
        L.oc_encode_cdf.argtypes = [vp, i64, vp, i64, i32, vp, i64]
        L.oc_dec_init.argtypes = [vp, vp, i64]
        L.oc_dec_symbol.restype = i32
        L.oc_dec_symbol.argtypes = [vp, vp, i32, i32]
        L.oc_decode_cdf.argtypes = [vp, i64, vp, i64, i64, i32, i32, vp]
        L.oc_dec_size.restype = i32
        L.oc_softmax_parts.argtypes = [vp, i32, vp, vp]
        L.oc_float_to_half.restype = C.c_uint16
        L.oc_float_to_half.argtypes = [C.c_float]
        _lib = L
    return _lib


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


def expf(x) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32).ravel()
    f = lib().oc_expf
    return np.array([f(float(v)) for v in x], dtype=np.float32)


def _threads(rows: int) -> int:
    return max(1, min(rows, os.cpu_count() or 1))


def cdf_from_logits(logits: np.ndarray, bits: int, threads: int | None = None) -> np.ndarray:
    """fp16 logits [rows, V] -> int32 CDF [rows, V+1] (cumulative)."""
    x = np.ascontiguousarray(logits, dtype=np.float16)
    if x.ndim == 1:
        x = x[None]
    rows, V = x.shape
    out = np.empty((rows, V + 1), dtype=np.int32)
    L = lib()
    nt = threads or _threads(rows)
    bounds = np.linspace(0, rows, nt + 1).astype(int)

    def work(i):
        a, b = int(bounds[i]), int(bounds[i + 1])
        if b > a:
            L.oc_cdf_from_logits(_p(x) + a * V * 2, V, b - a, V, bits, _p(out) + a * (V + 1) * 4)

    with cf.ThreadPoolExecutor(nt) as ex:
        list(ex.map(work, range(nt)))
    return out


def lohi_from_logits(logits: np.ndarray, symbols: np.ndarray, bits: int,
                     threads: int | None = None) -> np.ndarray:
    """(cdf[s], cdf[s+1]) per row: uint32 [rows, 2]."""
    x = np.ascontiguousarray(logits, dtype=np.float16)
    s = np.ascontiguousarray(symbols, dtype=np.int32).ravel()
    rows, V = x.shape
    out = np.empty((rows, 2), dtype=np.uint32)
    L = lib()
    nt = threads or _threads(rows)
    bounds = np.linspace(0, rows, nt + 1).astype(int)

    def work(i):
        a, b = int(bounds[i]), int(bounds[i + 1])
        if b > a:
            L.oc_lohi_from_logits(_p(x) + a * V * 2, V, b - a, V, bits, _p(s) + a * 4,
                                  _p(out) + a * 8)

    with cf.ThreadPoolExecutor(nt) as ex:
        list(ex.map(work, range(nt)))
    return out


SUBTILE = 32


def softmax_parts(logits: np.ndarray):
    """Per 32-column subtile: fp16 numerators e = fp16(e^(x - m_u)) (0 past V,
    shape [rows, nsub*64]) and partials (m_u, s_u) float32 [rows, nsub, 2] —
    what the head GEMM epilogue writes."""
    x = np.ascontiguousarray(logits, dtype=np.float16)
    if x.ndim == 1:
        x = x[None]
    rows, V = x.shape
    nsub = (V + SUBTILE - 1) // SUBTILE
    e16 = np.empty((rows, nsub * SUBTILE), dtype=np.float16)
    ms = np.empty((rows, nsub, 2), dtype=np.float32)
    for r in range(rows):
        lib().oc_softmax_parts(_p(x) + r * V * 2, V, _p(e16) + r * nsub * SUBTILE * 2,
                               _p(ms) + r * nsub * 8)
    return e16, ms


def cdf_from_probs(probs: np.ndarray, bits: int) -> np.ndarray:
    p = np.ascontiguousarray(probs, dtype=np.float32)
    if p.ndim == 1:
        p = p[None]
    rows, V = p.shape
    out = np.empty((rows, V + 1), dtype=np.int32)
    lib().oc_cdf_from_probs(_p(p), rows, V, bits, _p(out))
    return out


def _bits_of(cdf: np.ndarray) -> int:
    T = int(cdf[0, -1])
    assert T > 0 and T & (T - 1) == 0, f"CDF total {T} is not a power of two"
    return T.bit_length() - 1


def encode(cdf: np.ndarray, symbols: np.ndarray) -> bytes:
    """cpu_reference.encode: uint32 CDF [N, V+1] + symbols [N] -> bytes."""
    c = np.ascontiguousarray(cdf, dtype=np.uint32)
    s = np.ascontiguousarray(symbols, dtype=np.int32)
    N = c.shape[0]
    if N == 0:
        return bytes(encode_lohi(np.zeros((0, 2), np.uint32), 16))
    bits = _bits_of(c)
    cap = N * 8 + 64
    out = np.zeros(cap, dtype=np.uint8)
    n = lib().oc_encode_cdf(_p(c), c.shape[1], _p(s), N, bits, _p(out), cap)
    assert n >= 0, "oracle encode overflow"
    return out[:n].tobytes()


def encode_lohi(lohi: np.ndarray, bits: int) -> bytes:
    iv = np.ascontiguousarray(lohi, dtype=np.uint32).reshape(-1, 2)
    cap = iv.shape[0] * 8 + 64
    out = np.zeros(cap, dtype=np.uint8)
    n = lib().oc_encode_lohi(_p(iv), iv.shape[0], bits, _p(out), cap)
    assert n >= 0, "oracle encode overflow"
    return out[:n].tobytes()


class RangeDecoder:
    """cpu_reference.RangeDecoder: stateful, one CDF row per symbol."""

    def __init__(self, bitstream: bytes):
        self._buf = np.frombuffer(bytes(bitstream) or b"\0", dtype=np.uint8).copy()
        self._len = len(bitstream)
        self._st = (C.c_char * lib().oc_dec_size())()
        lib().oc_dec_init(C.addressof(self._st), _p(self._buf), self._len)

    def decode_symbol(self, cdf_row) -> int:
        row = np.ascontiguousarray(cdf_row, dtype=np.uint32)
        V = row.shape[0] - 1
        bits = int(row[-1]).bit_length() - 1
        return lib().oc_dec_symbol(C.addressof(self._st), _p(row), V, bits)


def decode(bitstream: bytes, cdfs: np.ndarray) -> np.ndarray:
    c = np.ascontiguousarray(cdfs, dtype=np.uint32)
    N, Vp1 = c.shape
    out = np.empty(N, dtype=np.int32)
    if N == 0:
        return out
    buf = np.frombuffer(bytes(bitstream) or b"\0", dtype=np.uint8).copy()
    lib().oc_decode_cdf(_p(buf), len(bitstream), _p(c), Vp1, N, Vp1 - 1, _bits_of(c), _p(out))
    return out
