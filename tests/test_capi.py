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


def test_lean_program_rule():
    """aicas_lean_program_ok: whole 2048-column chunks, k == 2048, or k == 6144
    with <= 2 row groups of 8 per CTA (not GATEUP); attention always passes."""
    L = _native.lib()

    def ph(kind, n, k):
        p = _native.AicasPhase()
        p.kind, p.n, p.k = kind, n, k
        return p

    def ok(*phases, nct=148):
        arr = (_native.AicasPhase * len(phases))(*phases)
        return L.aicas_lean_program_ok(arr, len(phases), nct)

    assert ok(ph(_native.PH_GEMV, 4096, 2048), ph(_native.PH_ATTN, 0, 0), ph(_native.PH_GATEUP, 6144, 2048),
              ph(_native.PH_GEMV, 2048, 6144), ph(_native.PH_LMHEAD, 151936, 2048)) == 0
    assert ok(ph(_native.PH_GEMV, 2048, 6144), nct=100) == 2      # 256 groups: 3 per CTA on 100 CTAs
    assert ok(ph(_native.PH_GEMV, 64, 4096)) == 2                 # two chunks
    assert ok(ph(_native.PH_GEMV, 64, 1024)) == 2                 # part of a chunk
    assert ok(ph(_native.PH_GATEUP, 64, 6144)) == 2
    assert ok(ph(_native.PH_LMHEAD, 64, 6144)) == 2               # the LM head: one chunk only
    assert ok(ph(_native.PH_GEMV, 64, 2048), nct=0) == 1


def test_prefill_attention_workspace_bytes():
    """The prefill attention's workspace: q rows and cache slots [0, start +
    rows) of every head in 128-row tiles, fp16; 0 for an invalid shape."""
    L = _native.lib()
    r128 = lambda x: (x + 127) // 128 * 128  # noqa: E731
    for rows, start, hq, hkv in [(1, 0, 16, 8), (1024, 0, 16, 8), (300, 0, 16, 8), (100, 200, 16, 8), (5, 3, 2, 1)]:
        want = (hq * r128(rows) + 2 * hkv * r128(start + rows)) * 128 * 2
        assert L.aicas_prefill_attention_workspace_bytes(rows, start, hq, hkv) == want
    assert L.aicas_prefill_attention_workspace_bytes(0, 0, 16, 8) == 0
    assert L.aicas_prefill_attention_workspace_bytes(4, -1, 16, 8) == 0
