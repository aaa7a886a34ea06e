"""The C-ABI library loads on a CPU host and exports every declared entry point."""
import ctypes
import re
from pathlib import Path

from krunch_b200 import _native as N

HDR = Path(__file__).resolve().parents[1] / "include"


def declared_symbols():
    names = set()
    for h in HDR.glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(kb_[a-z0-9_]+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    lib = N.load()
    decl = declared_symbols()
    assert len(decl) >= 20
    missing = [n for n in sorted(decl) if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_binding_covers_header():
    assert declared_symbols() == set(N.SIGNATURES)


def test_host_only_calls():
    lib = N.load()
    assert b"sm_100a" in lib.kb_version()
    assert lib.kb_status_string(0) == b"ok"
    assert lib.kb_status_string(-2) == b"unsupported shape"
    # argument validation happens before any device work
    assert lib.kb_gemm(0, None, 0, None, 0, 1, 128, 64, 0, None, 128, None, None, None) == -1
    assert lib.kb_cdf_rows(None, 0, 1, 10, 16, 0, None, 0, None, None, None) == -1
    assert lib.kb_coder_encode_lohi(None, 1, 1, None, 16, None, 0, None, None, None) == -1
    h = ctypes.c_void_p()
    d = N.ModelDesc()
    d.n_layer = 0
    assert lib.kb_model_create(ctypes.byref(d), ctypes.byref(h)) == -1
    assert lib.kb_forward_workspace_bytes(None, 1, 1) == 0
    assert lib.kb_layer_forward(None, 0, None, 1, 1, None, None, 0, None) == -1
    assert lib.kb_gemm_kvr(0, None, None, None, 768, None, None, None, None, None, None, 768,
                           None, None, None, 1, 768, 768, None, None, None, 768, 0, None) == -1
