"""CPU checks of the C ABI: the library loads, exports every symbol declared
in include/aicas_decode.h with the arity the ctypes binding uses, and its
struct layouts match the Python mirrors.  No kernel is launched."""
import re
from pathlib import Path


import _native

HEADER = Path(__file__).resolve().parent.parent / "include" / "aicas_decode.h"


def _declared():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    out = {}
    for m in re.finditer(r"AICAS_API\s+[\w\s\*]+?\b(aicas_\w+)\s*\(([^)]*)\)\s*;", text):
        args = [a for a in m.group(2).split(",") if a.strip() and a.strip() != "void"]
        out[m.group(1)] = len(args)
    return out


def test_header_declares_exports():
    decl = _declared()
    assert len(decl) >= 14
    assert set(decl) == set(_native.SIGNATURES), set(decl) ^ set(_native.SIGNATURES)
    for name, n in decl.items():
        assert len(_native.SIGNATURES[name][1]) == n, name


def test_library_exports_every_declared_symbol():
    L = _native.lib()
    for name in _declared():
        assert hasattr(L, name), name


def test_layouts_and_versions():
    L = _native.lib()
    assert L.aicas_abi_version() == 1
    assert _native.scratch_bytes() > 1_000_000
    assert L.aicas_error_string(10).decode().startswith("device:")
    assert L.aicas_error_string(0).decode() == "ok"


def test_host_validation_rejects_bad_phases():
    import ctypes

    L = _native.lib()
    p = _native.AicasPhase()
    p.kind = _native.PH_GEMV
    p.n, p.k = 16, 100  # k not a multiple of 8
    p.w = p.x = p.out = 4096
    arr = (_native.AicasPhase * 1)(p)
    assert L.aicas_validate_phases(arr, 1) == 2  # AICAS_ERR_SHAPE
    arr[0].k = 128
    arr[0].w = 4100  # misaligned
    assert L.aicas_validate_phases(arr, 1) == 3  # AICAS_ERR_ALIGN
    arr[0].w = 4096
    assert L.aicas_validate_phases(arr, 1) == 0
    arr[0].kind = 99
    assert L.aicas_validate_phases(arr, 1) == 1
    a = _native.AicasPhase()
    a.kind = _native.PH_ATTN
    a.kv_heads, a.q_heads, a.max_len = 8, 12, 64  # GQA ratio must be 2
    a.k_cache = a.v_cache = a.x = a.out = 4096
    assert L.aicas_validate_phases((_native.AicasPhase * 1)(a), 1) == 2
    del ctypes
