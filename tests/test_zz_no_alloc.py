"""The allocation-free attention entry point.

Some callers of this library cannot allocate device memory themselves (a
host framework that owns every allocation, a plugin that is only handed one
call's tensors), so `aicas_decode_attn_splitkv_f16_noalloc` keeps its scratch
in a fixed array inside the library.  These tests call it through the C ABI
and check that it returns what the scratch-taking entry point returns, on two
calls in a row (the second call reuses the array the first one left behind).
This file sorts last so a run that stops at the first failure has already run
every other test.
"""
import ctypes

import pytest
import torch

import _native

pytestmark = pytest.mark.gpu

ATOL = 2e-3  # the attention tolerance of tests/test_ops_gpu.py


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def test_noalloc_attention_matches_scratch_entry_point(cuda_device):
    L = _native.lib()
    lmax = 8192
    g = torch.Generator().manual_seed(2024)
    q = torch.randn(16 * 128, generator=g).half().to(cuda_device)
    k = torch.randn((8, lmax, 128), generator=g).half().to(cuda_device)
    v = torch.randn((8, lmax, 128), generator=g).half().to(cuda_device)
    scratch = torch.zeros(_native.scratch_bytes(), dtype=torch.uint8, device=cuda_device)
    status = torch.full((1,), -1, dtype=torch.int32, device=cuda_device)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for valid in (777, 4096):
        pos = torch.tensor([valid - 1], dtype=torch.int64, device=cuda_device)
        ref = torch.empty(16 * 128, dtype=torch.float16, device=cuda_device)
        got = torch.empty_like(ref)
        rc = L.aicas_decode_attn_splitkv_f16(_p(q), _p(k), _p(v), _p(pos), 128 ** -0.5, _p(ref), 16, 8, lmax,
                                             _p(scratch), stream)
        _native.check(rc, "aicas_decode_attn_splitkv_f16")
        rc = L.aicas_decode_attn_splitkv_f16_noalloc(_p(q), _p(k), _p(v), _p(pos), 128 ** -0.5, _p(got), 16, 8,
                                                     lmax, _p(status), stream)
        _native.check(rc, "aicas_decode_attn_splitkv_f16_noalloc")
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert float((got.float() - ref.float()).abs().max()) <= ATOL


def test_noalloc_rejects_more_heads_than_its_scratch_holds(cuda_device):
    L = _native.lib()
    t = torch.zeros(8, dtype=torch.float16, device=cuda_device)
    pos = torch.zeros(1, dtype=torch.int64, device=cuda_device)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = L.aicas_decode_attn_splitkv_f16_noalloc(_p(t), _p(t), _p(t), _p(pos), 0.1, _p(t), 32, 16, 64, None, stream)
    assert rc == 5  # AICAS_ERR_CAPACITY, rejected on the host before any launch
    assert "fixed device scratch" in _native.error_message(rc)
