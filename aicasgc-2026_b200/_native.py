"""ctypes binding of `libaicas_decode.so`, the C ABI declared in
`include/aicas_decode.h`.

The library is built in-tree for sm_100a by `build_native.py`.  There is no
fallback: importing an op wrapper on a machine without the built library, or
calling it without a CUDA device, raises.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("AICAS_LIB", str(HERE / "libaicas_decode.so")))

# Phase kinds / flags (include/aicas_phase_program.h)
PH_GEMV, PH_GATEUP, PH_ATTN, PH_LMHEAD = 1, 2, 3, 4
PROGRAM_LEAN = 1  # aicas_decode_program_ex_f16 flag: the lean kernel instantiation
F_NORM = 1 << 0
F_X_EMBED = 1 << 1
F_RESID = 1 << 2
F_RESID_EMBED = 1 << 3
F_BIAS = 1 << 4
F_X_ADD = 1 << 5
F_RESID_ADD = 1 << 6
F_Q_READY = 1 << 7
F_STORE_X = 1 << 8
F_KBLOCKED = 1 << 9
F_BARRIER = 1 << 10
F_LL_IN = 1 << 11
F_LL_OUT = 1 << 12
F_LL_RESID = 1 << 13
F_CNT_IN = 1 << 14
F_CNT_OUT = 1 << 15
F_CNT_RESID = 1 << 16

DEVICE_ERRORS = {
    10: "grid barrier timed out",
    11: "bulk copy did not complete in time",
    12: "ring stage was not released in time",
    13: "in-flight copies did not drain in time",
    14: "bad phase descriptor",
    15: "token id or cache position out of range",
    16: "an input vector did not arrive in time",
    17: "a tensor-memory slot hand-off did not complete in time",
}


class AicasError(RuntimeError):
    pass


class AicasPhase(ctypes.Structure):
    _fields_ = [
        ("kind", ctypes.c_int32), ("flags", ctypes.c_int32), ("n", ctypes.c_int32), ("k", ctypes.c_int32),
        ("rot", ctypes.c_int32), ("kv_heads", ctypes.c_int32), ("q_heads", ctypes.c_int32),
        ("max_len", ctypes.c_int32), ("embed_rows", ctypes.c_int32), ("x_src", ctypes.c_int32),
        ("w", ctypes.c_void_p), ("norm_w", ctypes.c_void_p), ("norm_w2", ctypes.c_void_p),
        ("x", ctypes.c_void_p), ("x2", ctypes.c_void_p), ("resid", ctypes.c_void_p),
        ("resid2", ctypes.c_void_p), ("bias", ctypes.c_void_p), ("out", ctypes.c_void_p),
        ("x_out", ctypes.c_void_p), ("k_cache", ctypes.c_void_p), ("v_cache", ctypes.c_void_p),
        ("pos_ptr", ctypes.c_void_p), ("idx_out", ctypes.c_void_p),
        ("eps", ctypes.c_float), ("scale", ctypes.c_float),
    ]


class AicasStepState(ctypes.Structure):
    _fields_ = [
        ("token", ctypes.c_int64), ("cache_pos", ctypes.c_int64), ("rope", ctypes.c_int64 * 3),
        ("step", ctypes.c_int64), ("script_len", ctypes.c_int64), ("script", ctypes.c_void_p),
        ("out_tokens", ctypes.c_void_p), ("max_steps", ctypes.c_int64), ("logits", ctypes.c_void_p),
        ("logits_ring", ctypes.c_int64), ("inv_freq", ctypes.c_float * 64),
        ("mrope_section", ctypes.c_int32 * 3), ("pad0", ctypes.c_int32),
        ("eos_token", ctypes.c_int64), ("done_step", ctypes.c_int64),
    ]


# Streams of one batched launch (AICAS_MAX_BATCH).
MAX_BATCH = 8

# Offsets of the scratch words the host reads (AicasScratch; the batch
# scratch block starts with the same words).
SCRATCH_ERROR_OFFSET = 16

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_F = ctypes.c_float
_I = ctypes.c_int

# exported symbol -> (restype, argtypes); the tests check this list against
# the declarations in include/aicas_decode.h.
SIGNATURES = {
    "aicas_abi_version": (_I, []),
    "aicas_error_string": (ctypes.c_char_p, [_I]),
    "aicas_last_cuda_error": (_I, []),
    "aicas_cuda_error_string": (ctypes.c_char_p, [_I]),
    "aicas_scratch_bytes": (ctypes.c_size_t, []),
    "aicas_layout_signature": (_I, [ctypes.POINTER(_I64), _I]),
    "aicas_num_ctas": (_I, [_I]),
    "aicas_set_cooperative_launch": (_I, [_I]),
    "aicas_validate_phases": (_I, [ctypes.POINTER(AicasPhase), _I]),
    "aicas_gemv_f16": (_I, [_P, _P, _P, _P, _I64, _I64, _P, _P]),
    "aicas_rmsnorm_qkv_f16": (_I, [_P, _P, _P, _P, _P, _I64, _I64, _F, _P, _P]),
    "aicas_post_attn_mlp_f16": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _F, _P, _P]),
    "aicas_decode_attn_splitkv_f16": (_I, [_P, _P, _P, _P, _F, _P, _I64, _I64, _I64, _P, _P]),
    "aicas_decode_attn_splitkv_f16_noalloc": (_I, [_P, _P, _P, _P, _F, _P, _I64, _I64, _I64, _P, _P]),
    "aicas_qk_norm_mrope_kvwrite_f16": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _F, _I64, _I64, _I64, _P]),
    "aicas_lm_head_argmax_f16": (_I, [_P, _P, _P, _P, _P, _I64, _I64, _F, _P, _P]),
    "aicas_decode_program_f16": (_I, [_P, _I, _P, _P, _P]),
    "aicas_decode_program_trace_f16": (_I, [_P, _I, _P, _P, _P, _P]),
    "aicas_lean_program_ok": (_I, [ctypes.POINTER(AicasPhase), _I, _I]),
    "aicas_decode_program_ex_f16": (_I, [_P, _I, _P, _P, _P, _I, _P]),
    "aicas_batch_scratch_bytes": (ctypes.c_size_t, []),
    "aicas_validate_batch_phases": (_I, [ctypes.POINTER(AicasPhase), _I]),
    "aicas_decode_batch_f16": (_I, [_P, _I, _P, _I, _P, _P]),
    "aicas_decode_batch_trace_f16": (_I, [_P, _I, _P, _I, _P, _P, _P]),
    "aicas_tile_weight_f16": (_I, [_P, _P, _I64, _I64, _P]),
    "aicas_prefill_add_rmsnorm_f16": (_I, [_P, _P, _P, _P, _P, _I64, _I64, _F, _P]),
    "aicas_prefill_qk_norm_rope_kv_f16": (_I, [_P, _P, _P, _P, _P, _I, _I, _P, _P, _P, _I64, _I64, _I64, _I64,
                                               _I64, _F, _P, _P]),
    "aicas_prefill_silu_mul_f16": (_I, [_P, _P, _I64, _I64, _P]),
    "aicas_prefill_attention_workspace_bytes": (ctypes.c_size_t, [_I64, _I64, _I64, _I64]),
    "aicas_prefill_attention_f16": (_I, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _F, _P, _P]),
    "aicas_prefill_attention_tiles_f16": (_I, [_P, _P, _I64, _I64, _I64, _I64, _F, _P]),
    "aicas_prefill_attention_timeouts": (_I, []),
}

_lock = threading.Lock()
_lib = None


def lib() -> ctypes.CDLL:
    """Load the native library once and check its ABI and struct layouts."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise AicasError(f"{LIB_PATH.name} is not built; run build_native.py (nvcc, sm_100a)")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        if L.aicas_abi_version() != 1:
            raise AicasError("ABI version mismatch")
        sig = (ctypes.c_int64 * 8)()
        n = L.aicas_layout_signature(sig, 8)
        want = [ctypes.sizeof(AicasPhase), ctypes.sizeof(AicasStepState), None,
                AicasPhase.w.offset, AicasPhase.eps.offset, AicasStepState.inv_freq.offset, None,
                SCRATCH_ERROR_OFFSET]
        for i in range(min(n, len(want))):
            if want[i] is not None and sig[i] != want[i]:
                raise AicasError(f"struct layout mismatch at {i}: lib {sig[i]} vs ctypes {want[i]}")
        _lib = L
        return L


def check(rc: int, what: str) -> None:
    if rc != 0:
        L = lib()
        msg = L.aicas_error_string(rc).decode()
        if rc == 4:  # AICAS_ERR_CUDA
            ce = L.aicas_last_cuda_error()
            msg += f": {L.aicas_cuda_error_string(ce).decode()} (cudaError {ce})"
        raise AicasError(f"{what} failed: {msg} (code {rc})")


def scratch_bytes() -> int:
    return int(lib().aicas_scratch_bytes())


def batch_scratch_bytes() -> int:
    return int(lib().aicas_batch_scratch_bytes())


def error_message(code: int) -> str:
    return lib().aicas_error_string(int(code)).decode()
