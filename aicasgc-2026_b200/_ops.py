"""Torch-tensor front end of the C ABI: argument checks, output allocation,
per-device scratch blocks, device-error reporting.

Every call goes to `libaicas_decode.so`; there is no CPU or eager-PyTorch
fallback.  Tensors must be CUDA fp16 (cache positions int64), contiguous.
"""
from __future__ import annotations

import ctypes

import torch

from _native import (DEVICE_ERRORS, SCRATCH_ERROR_OFFSET, AicasError, check, lib,
                     scratch_bytes)

_scratch: dict[tuple[int, int], torch.Tensor] = {}


def scratch_for(device: torch.device) -> torch.Tensor:
    """The scratch block of `device`'s current stream (zero-filled once,
    reused by every op issued on that stream).  One block per stream: ops on
    one stream are ordered, so they never share a block concurrently, and ops
    on two streams never share one at all.  A device error recorded in a
    block makes every later op on that stream do nothing until
    `raise_if_device_error` (which zeroes the block) is called."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, torch.cuda.current_stream(idx).cuda_stream)
    t = _scratch.get(key)
    if t is None:
        t = torch.zeros(scratch_bytes(), dtype=torch.uint8, device=torch.device("cuda", idx))
        _scratch[key] = t
    return t


def device_error(scratch: torch.Tensor) -> int:
    """Error word of a scratch block (synchronises the current stream)."""
    return int(scratch[SCRATCH_ERROR_OFFSET:SCRATCH_ERROR_OFFSET + 4].view(torch.int32).item())


def raise_if_device_error(scratch: torch.Tensor) -> None:
    code = device_error(scratch)
    if code:
        scratch.zero_()
        raise AicasError(f"device error {code}: {DEVICE_ERRORS.get(code, 'unknown')}")


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _need(cond: bool, msg: str):
    if not cond:
        raise AicasError(msg)


def _f16(t: torch.Tensor, name: str):
    _need(t.is_cuda and t.dtype == torch.float16, f"{name} must be a CUDA fp16 tensor")
    _need(t.is_contiguous(), f"{name} must be contiguous")


def gemv(x: torch.Tensor, w: torch.Tensor, bias=None, out=None, norm_w=None, eps: float = 1e-6):
    """out[n] = W[n,k] @ (RMSNorm(x) if norm_w else x) (+ bias)."""
    _f16(w, "weight")
    _need(w.dim() == 2, "weight must be [n, k]")
    n, k = w.shape
    xv = x.reshape(-1)
    _f16(xv, "x")
    _need(xv.numel() == k, f"x has {xv.numel()} elements, weight expects {k}")
    if bias is not None:
        _f16(bias, "bias")
    if out is None:
        out = torch.empty(n, dtype=torch.float16, device=w.device)
    sc = scratch_for(w.device)
    if norm_w is None:
        rc = lib().aicas_gemv_f16(_ptr(xv), _ptr(w), _ptr(bias), _ptr(out), n, k, _ptr(sc), _stream())
        check(rc, "aicas_gemv_f16")
    else:
        _f16(norm_w, "norm_weight")
        rc = lib().aicas_rmsnorm_qkv_f16(_ptr(xv), _ptr(norm_w), _ptr(w), _ptr(bias), _ptr(out), n, k,
                                         float(eps), _ptr(sc), _stream())
        check(rc, "aicas_rmsnorm_qkv_f16")
    return out


def post_attn_mlp(residual, attn_out, norm_w, gate_up_w, down_w, bias=None, eps=1e-6, act_out=None, out=None):
    for t, nm in ((gate_up_w, "gate_up_weight"), (down_w, "down_proj_weight"), (norm_w, "norm_weight")):
        _f16(t, nm)
    r = residual.reshape(-1)
    a = attn_out.reshape(-1)
    _f16(r, "residual")
    _f16(a, "attn_output")
    hidden, inter = down_w.shape
    _need(gate_up_w.shape == (2 * inter, hidden), "gate_up weight must be [2*inter, hidden]")
    _need(r.numel() == hidden and a.numel() == hidden, "residual/attn_output size mismatch")
    if act_out is None:
        act_out = torch.empty(inter, dtype=torch.float16, device=r.device)
    if out is None:
        out = torch.empty(hidden, dtype=torch.float16, device=r.device)
    sc = scratch_for(r.device)
    rc = lib().aicas_post_attn_mlp_f16(_ptr(r), _ptr(a), _ptr(norm_w), _ptr(gate_up_w), _ptr(down_w),
                                       _ptr(bias), _ptr(act_out), _ptr(out), hidden, inter, float(eps),
                                       _ptr(sc), _stream())
    check(rc, "aicas_post_attn_mlp_f16")
    return act_out, out


def decode_attention(q, k_cache, v_cache, cache_position, scale, out=None):
    """q [Hq,128] (any shape with Hq*128 elements), K/V [KVH, Lmax, 128]."""
    _f16(k_cache, "k_cache")
    _f16(v_cache, "v_cache")
    qv = q.reshape(-1)
    _f16(qv, "q")
    _need(cache_position.is_cuda and cache_position.dtype == torch.int64, "cache_position must be CUDA int64")
    kvh, lmax, hd = k_cache.shape[-3:]
    _need(hd == 128 and k_cache.shape == v_cache.shape, "cache must be [.., KVH, Lmax, 128]")
    hq = qv.numel() // 128
    if out is None:
        out = torch.empty(hq * 128, dtype=torch.float16, device=qv.device)
    sc = scratch_for(qv.device)
    rc = lib().aicas_decode_attn_splitkv_f16(_ptr(qv), _ptr(k_cache), _ptr(v_cache), _ptr(cache_position),
                                             float(scale), _ptr(out), hq, kvh, lmax, _ptr(sc), _stream())
    check(rc, "aicas_decode_attn_splitkv_f16")
    return out


def qk_norm_rope_kvwrite(q, k, v, q_norm_w, k_norm_w, cos, sin, k_cache, v_cache, cache_position, eps,
                         q_out=None):
    for t, nm in ((q, "q"), (k, "k"), (v, "v"), (q_norm_w, "q_weight"), (k_norm_w, "k_weight"),
                  (cos, "cos"), (sin, "sin"), (k_cache, "k_cache"), (v_cache, "v_cache")):
        _f16(t, nm)
    _need(cache_position.is_cuda and cache_position.dtype == torch.int64, "cache_position must be CUDA int64")
    kvh, lmax, hd = k_cache.shape[-3:]
    hq = q.numel() // 128
    if q_out is None:
        q_out = torch.empty_like(q)
    rc = lib().aicas_qk_norm_mrope_kvwrite_f16(_ptr(q), _ptr(k), _ptr(v), _ptr(q_norm_w), _ptr(k_norm_w),
                                               _ptr(cos), _ptr(sin), _ptr(q_out), _ptr(k_cache),
                                               _ptr(v_cache), _ptr(cache_position), float(eps), hq, kvh,
                                               lmax, _stream())
    check(rc, "aicas_qk_norm_mrope_kvwrite_f16")
    return q_out


def lm_head_argmax(x, w, norm_w=None, eps=1e-6, logits=None, token_out=None, want_logits=True):
    _f16(w, "weight")
    xv = x.reshape(-1)
    _f16(xv, "x")
    vocab, k = w.shape
    if want_logits and logits is None:
        logits = torch.empty(vocab, dtype=torch.float16, device=w.device)
    if token_out is None:
        token_out = torch.empty(1, dtype=torch.int64, device=w.device)
    sc = scratch_for(w.device)
    rc = lib().aicas_lm_head_argmax_f16(_ptr(xv), _ptr(norm_w), _ptr(w), _ptr(logits), _ptr(token_out),
                                        vocab, k, float(eps), _ptr(sc), _stream())
    check(rc, "aicas_lm_head_argmax_f16")
    return logits, token_out
