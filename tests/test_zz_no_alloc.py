"""The allocation-free attention entry point.

Some callers of this library cannot allocate device memory themselves (a
host framework that owns every allocation, a plugin that is only handed one
call's tensors), so `aicas_decode_attn_splitkv_f16_noalloc` keeps its scratch
in a fixed array inside the library.  These tests call it through the C ABI
and check that it returns exactly what the scratch-taking entry point returns
on several calls in a row (each call reuses the array the previous one left
behind, longer and shorter contexts alike, and after a call that ended with a
device error).
This file sorts last so a run that stops at the first failure has already run
every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

import _native
from oracle.qwen3vl_oracle import attention_reference

pytestmark = pytest.mark.gpu

ATOL = 2e-3  # the attention tolerance of tests/test_ops_gpu.py (against the fp32 reference)
K_ERR_BAD_INPUT = 15


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _inputs(dev, lmax=8192):
    g = torch.Generator().manual_seed(2024)
    q = torch.randn(16 * 128, generator=g).half().to(dev)
    k = torch.randn((8, lmax, 128), generator=g).half().to(dev)
    v = torch.randn((8, lmax, 128), generator=g).half().to(dev)
    return q, k, v


def _both(L, q, k, v, valid, lmax, scratch, status, stream):
    """The scratch-taking entry point and the allocation-free one on the same
    inputs; returns (scratch result, allocation-free result)."""
    dev = q.device
    pos = torch.tensor([valid - 1], dtype=torch.int64, device=dev)
    ref = torch.empty(16 * 128, dtype=torch.float16, device=dev)
    got = torch.full_like(ref, float("nan"))
    rc = L.aicas_decode_attn_splitkv_f16(_p(q), _p(k), _p(v), _p(pos), 128 ** -0.5, _p(ref), 16, 8, lmax,
                                         _p(scratch), stream)
    _native.check(rc, "aicas_decode_attn_splitkv_f16")
    rc = L.aicas_decode_attn_splitkv_f16_noalloc(_p(q), _p(k), _p(v), _p(pos), 128 ** -0.5, _p(got), 16, 8,
                                                 lmax, _p(status), stream)
    _native.check(rc, "aicas_decode_attn_splitkv_f16_noalloc")
    torch.cuda.synchronize()
    return ref, got


def test_noalloc_attention_matches_scratch_entry_point(cuda_device):
    """Calls in a row on the shared array, long then short then long again:
    each result is bit-identical to the scratch-taking entry point's (the
    same deterministic kernel) and within the op tolerance of the fp32
    attention reference."""
    L = _native.lib()
    lmax = 8192
    q, k, v = _inputs(cuda_device, lmax)
    scratch = torch.zeros(_native.scratch_bytes(), dtype=torch.uint8, device=cuda_device)
    status = torch.full((1,), -1, dtype=torch.int32, device=cuda_device)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for valid in (777, 4096, 777, 8192):
        ref, got = _both(L, q, k, v, valid, lmax, scratch, status, stream)
        assert int(status.item()) == 0
        assert torch.equal(got, ref), f"valid {valid}: not bit-identical to the scratch entry point"
        exp = attention_reference(q.view(16, 128).float().cpu().numpy(), k[:, :valid].float().cpu().numpy(),
                                  v[:, :valid].float().cpu().numpy(), valid, 128 ** -0.5)
        assert np.abs(got.view(16, 128).float().cpu().numpy() - exp).max() <= ATOL


def test_noalloc_device_error_then_a_good_call(cuda_device):
    """A cache position outside the cache is found on the device (no read past
    the cache, no fault) and reported through `status`; the next call starts
    from a cleared error word and matches the scratch entry point again."""
    L = _native.lib()
    lmax = 1024
    q, k, v = _inputs(cuda_device, lmax)
    status = torch.full((1,), -1, dtype=torch.int32, device=cuda_device)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    bad = torch.tensor([lmax], dtype=torch.int64, device=cuda_device)  # slot == cache length
    out = torch.zeros(16 * 128, dtype=torch.float16, device=cuda_device)
    rc = L.aicas_decode_attn_splitkv_f16_noalloc(_p(q), _p(k), _p(v), _p(bad), 128 ** -0.5, _p(out), 16, 8, lmax,
                                                 _p(status), stream)
    _native.check(rc, "aicas_decode_attn_splitkv_f16_noalloc")
    torch.cuda.synchronize()
    assert int(status.item()) == K_ERR_BAD_INPUT
    scratch = torch.zeros(_native.scratch_bytes(), dtype=torch.uint8, device=cuda_device)
    ref, got = _both(L, q, k, v, 500, lmax, scratch, status, stream)
    assert int(status.item()) == 0
    assert torch.equal(got, ref)


def test_noalloc_rejects_more_heads_than_its_scratch_holds(cuda_device):
    L = _native.lib()
    t = torch.zeros(8, dtype=torch.float16, device=cuda_device)
    pos = torch.zeros(1, dtype=torch.int64, device=cuda_device)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = L.aicas_decode_attn_splitkv_f16_noalloc(_p(t), _p(t), _p(t), _p(pos), 0.1, _p(t), 32, 16, 64, None, stream)
    assert rc == 5  # AICAS_ERR_CAPACITY, rejected on the host before any launch
    assert "fixed device scratch" in _native.error_message(rc)
