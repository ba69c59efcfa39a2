"""Drop-in for the reference's `cuda_decode_attention` module.

`decode_attn_v4_cta_qhead_splitkv_fused` keeps the signature, preconditions
(returns None when they fail, so callers fall through as in
`optimized_layer.py:2394-2415`) and output layout of
`cuda_decode_attention.py:489-558`.  As there, `split_k <= 1` returns None
(the reference's caller then runs its non-split attention).  Any larger
`split_k` and the `workspace` are accepted for compatibility: the B200 kernel
splits the cache over every SM itself and keeps its partials in the scratch
block of the calling stream.
"""
from __future__ import annotations

import torch

import _ops

__all__ = ["decode_attn_v4_cta_qhead_splitkv_fused"]


def decode_attn_v4_cta_qhead_splitkv_fused(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scaling: float,
                                           num_key_value_groups: int, cache_position: torch.Tensor,
                                           split_k: int = 4, workspace: dict | None = None):
    """q [1, Hq, 1, 128]; k/v [1, KVH, Lmax, 128] (HF StaticLayer layout);
    attends slots [0, cache_position]; returns [1, 1, Hq, 128]."""
    del workspace
    if (num_key_value_groups != 2 or split_k <= 1 or q.device.type != "cuda" or k.device.type != "cuda"
            or v.device.type != "cuda" or cache_position.device.type != "cuda" or q.shape[0] != 1
            or q.shape[2] != 1 or q.shape[-1] != 128 or q.dtype != torch.float16
            or k.dtype != torch.float16 or v.dtype != torch.float16
            or k.shape[1] * num_key_value_groups != q.shape[1] or k.shape[0] != 1
            or not k.is_contiguous() or not v.is_contiguous()):
        return None
    out = _ops.decode_attention(q.reshape(-1).contiguous(), k[0], v[0], cache_position.reshape(-1)[:1],
                                scaling)
    return out.view(1, 1, q.shape[1], 128)
