"""ctypes binding of libkrunch_b200.so (the C ABI declared in include/krunch_b200.h).

Loading fails loudly when the library is missing: there is no CPU fallback
for any entry point.  Tensor arguments are PyTorch CUDA tensors; this module
passes their data pointers and the current CUDA stream.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

_LIB_PATH = Path(os.environ.get("KRUNCH_B200_LIB", "") or Path(__file__).resolve().parent / "libkrunch_b200.so")  # override: another build of the library

KB_OK = 0
KB_ERR_TOO_LARGE = -9
KB_ERR_TIMEOUT = -5
KB_NOALLOC_SCRATCH_BYTES = 8 << 20
KB_CDF_COUNTS, KB_CDF_CDF, KB_CDF_LOHI = 0, 1, 2
KB_EPI_F32, KB_EPI_F16, KB_EPI_SIGMOID, KB_EPI_RELU_SQ, KB_EPI_RESID, KB_EPI_GATE_RESID = range(6)
KB_F16, KB_BF16, KB_I8 = 0, 1, 2
KB_TILE_PAIR = 512  # kb_gemm_tiled / kb_gemm_i8: CTA-pair 256 x 256 tiles
KB_WKV_STEP_REF, KB_WKV_PRODUCTION = 0, 1

vp = C.c_void_p
i32 = C.c_int
i64 = C.c_int64
sz = C.c_size_t


class LayerDesc(C.Structure):
    _fields_ = [(n, vp) for n in (
        "ln1_w", "ln1_b", "ln2_w", "ln2_b",
        "att_mix_k", "att_mix_v", "att_mix_r", "att_decay", "att_first",
        "att_kw", "att_vw", "att_rw", "att_ow",
        "ffn_mix_k", "ffn_mix_r", "ffn_kw", "ffn_vw", "ffn_rw",
        "att_ks", "att_vs", "att_rs", "att_os", "ffn_ks", "ffn_vs", "ffn_rs")]


class ModelDesc(C.Structure):
    _fields_ = [("n_layer", i32), ("n_embd", i32), ("n_ffn", i32), ("n_vocab", i32),
                ("vocab_pad", i32), ("wdtype", i32), ("wkv_convention", i32),
                ("emb", vp), ("ln_out_w", vp), ("ln_out_b", vp), ("head", vp),
                ("layers", C.POINTER(LayerDesc)), ("head_scale", vp)]


# name -> (restype, argtypes); mirrors include/krunch_b200.h
SIGNATURES = {
    "kb_version": (C.c_char_p, []),
    "kb_status_string": (C.c_char_p, [i32]),
    "kb_last_cuda_error": (i32, []),
    "kb_profile_begin": (i32, []),
    "kb_profile_end": (i32, [vp, vp, vp, i32]),
    "kb_coder_encode_init": (i32, [vp, i32, vp]),
    "kb_coder_encode_cdf": (i32, [vp, i64, vp, i32, i32, vp, i64, vp, vp]),
    "kb_coder_encode_cdf_batched": (i32, [vp, i64, vp, i32, i32, vp, i64, vp, vp, vp]),
    "kb_coder_encode_lohi": (i32, [vp, i32, i32, vp, i32, vp, i64, vp, vp, vp]),
    "kb_coder_encode_finalize": (i32, [vp, i64, vp, vp, i32, vp]),
    "kb_coder_decode_init": (i32, [vp, i64, vp, vp, i32, vp]),
    "kb_coder_decode_cdf": (i32, [vp, i64, i32, i32, vp, i64, vp, vp, vp, i32, vp]),
    "kb_cdf_rows": (i32, [vp, i64, i32, i32, i32, i32, vp, i64, vp, vp, vp]),
    "kb_cdf_from_probs": (i32, [vp, i32, i32, i32, vp, vp]),
    "kb_decode_logits_step": (i32, [vp, i64, i32, i32, i32, vp, i64, vp, i64, vp, vp, vp, vp, vp, i64, vp]),
    "kb_device_error_status": (i32, [i32]),
    "kb_gemm": (i32, [i32, vp, i64, vp, i64, i32, i32, i32, i32, vp, i64, vp, vp, vp]),
    "kb_step_workspace_bytes": (sz, [vp, i32]),
    "kb_step_forward": (i32, [vp, vp, i32, vp, vp, sz, vp, vp, vp]),
    "kb_step_error_status": (i32, [i32]),
    "kb_step_set_trace": (i32, [vp]),
    "kb_step_set_fault": (i32, [i32, i64]),
    "kb_gemm_i8": (i32, [vp, i64, vp, vp, i64, vp, i32, i32, i32, i32, vp, i64, vp, vp, i32, vp]),
    "kb_gemm_kvr": (i32, [i32, vp, vp, vp, i64, vp, vp, vp, vp, vp, vp, i64, vp, vp, vp, i32, i32,
                          i32, vp, vp, vp, i64, i32, vp]),
    "kb_quantize_weight": (i32, [vp, i32, i32, vp, vp, vp]),
    "kb_quantize_rows": (i32, [vp, i32, i32, vp, vp, vp]),
    "kb_gemm_tiled": (i32, [i32, vp, i64, vp, i64, i32, i32, i32, i32, vp, i64, vp, vp, i32, vp]),
    "kb_model_create": (i32, [C.POINTER(ModelDesc), C.POINTER(vp)]),
    "kb_model_destroy": (None, [vp]),
    "kb_prepare_decay": (i32, [vp, vp, i32, vp]),
    "kb_state_init": (i32, [vp, vp, i32, vp]),
    "kb_forward_workspace_bytes": (sz, [vp, i32, i32]),
    "kb_forward_window": (i32, [vp, vp, i32, i32, vp, vp, sz, vp, vp, vp]),
    "kb_layer_forward": (i32, [vp, i32, vp, i32, i32, vp, vp, sz, vp]),
    "kb_forward_window_noalloc": (i32, [vp, vp, i32, i32, vp, vp, vp]),
}

_lib = None


def lib_path() -> Path:
    return _LIB_PATH


def load() -> C.CDLL:
    """Load the native library (once).  Raises RuntimeError if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not _LIB_PATH.exists():
        raise RuntimeError(
            f"{_LIB_PATH} is missing: build it with `python -m krunch_b200.build` "
            "(krunch_b200 has no CPU fallback)")
    lib = C.CDLL(str(_LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


class KBError(RuntimeError):
    pass


def check(status: int, what: str) -> None:
    if status != KB_OK:
        lib = load()
        msg = lib.kb_status_string(status).decode()
        extra = ""
        if status == -4:
            extra = f" (cudaError {lib.kb_last_cuda_error()})"
        raise KBError(f"{what} failed: {msg}{extra}")


def ptr(t) -> int | None:
    """Data pointer of a tensor (None passes NULL)."""
    if t is None:
        return None
    return t.data_ptr()


def stream_ptr(device=None) -> int:
    import torch
    return torch.cuda.current_stream(device).cuda_stream


def call(name: str, *args) -> None:
    """Call an entry point and raise on a non-zero status."""
    lib = load()
    check(getattr(lib, name)(*args), name)


PHASES = ("embed", "ln_mix", "gemm", "wkv", "head", "cdf", "encode", "decode", "step")


def profile_begin() -> None:
    call("kb_profile_begin")


def profile_end() -> dict:
    """{phase: (ms, launches, work)} for launches since profile_begin()."""
    n = len(PHASES)
    ms, cnt, work = (C.c_double * n)(), (C.c_int64 * n)(), (C.c_double * n)()
    call("kb_profile_end", C.cast(ms, vp), C.cast(cnt, vp), C.cast(work, vp), n)
    return {p: (ms[i], cnt[i], work[i]) for i, p in enumerate(PHASES)}


def env_flag(name: str, default: str = "0") -> bool:
    return os.environ.get(name, default) not in ("0", "", "false", "False")
