"""Drop-in for the reference's `cuda_decode_small_ops` module.

`fused_q_rope_kv_cache_update` keeps the signature, checks and return value
of `cuda_decode_small_ops.py:136-225`: q/k per-head RMSNorm + RoPE with the
given cos/sin, k and v written into the static cache at `cache_position`,
rotated q returned.
"""
from __future__ import annotations

import torch

import _ops

__all__ = ["fused_q_rope_kv_cache_update"]


def fused_q_rope_kv_cache_update(q, k, v, q_weight, k_weight, eps, cos, sin, k_cache, v_cache, cache_position):
    ts = (q, k, v, q_weight, k_weight, cos, sin, k_cache, v_cache)
    if any(t.device.type != "cuda" for t in ts + (cache_position,)) or any(t.dtype != torch.float16 for t in ts) \
            or cache_position.dtype != torch.long:
        raise RuntimeError("fused_q_rope_kv_cache_update expects fp16 CUDA tensors and int64 cache_position")
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise RuntimeError("fused_q_rope_kv_cache_update expects q/k/v as [B, S, H, D]")
    if q.shape[:2] != k.shape[:2] or k.shape != v.shape:
        raise RuntimeError("q/k/v shapes must match decode layout")
    if q.shape[0] != 1 or q.shape[1] != 1:
        raise RuntimeError("fused_q_rope_kv_cache_update currently supports single-token decode only")
    if q.shape[-1] != 128 or k.shape[-1] != 128:
        raise RuntimeError("fused_q_rope_kv_cache_update currently supports only head_dim=128")
    if q.shape[2] != k.shape[2] * 2:
        raise RuntimeError("fused_q_rope_kv_cache_update currently supports q_heads == 2 * kv_heads")
    if q_weight.numel() != 128 or k_weight.numel() != 128:
        raise RuntimeError("fused_q_rope_kv_cache_update expects q/k norm weights of shape [128]")
    if cos.shape != q.shape[:2] + (128,) or sin.shape != q.shape[:2] + (128,):
        raise RuntimeError("fused_q_rope_kv_cache_update expects cos/sin shaped [B, S, 128]")
    if k_cache.ndim != 4 or k_cache.shape[0] != 1 or k_cache.shape[1] != k.shape[2] or k_cache.shape[-1] != 128:
        raise RuntimeError("fused_q_rope_kv_cache_update expects k_cache/v_cache as [1, KVH, T, 128]")
    if cache_position.ndim != 1 or cache_position.numel() != 1:
        raise RuntimeError("cache_position must be shape [1]")
    q_out = _ops.qk_norm_rope_kvwrite(q.contiguous(), k.contiguous(), v.contiguous(), q_weight.contiguous(),
                                      k_weight.contiguous(), cos.contiguous(), sin.contiguous(), k_cache,
                                      v_cache, cache_position, eps)
    return q_out.view_as(q)
