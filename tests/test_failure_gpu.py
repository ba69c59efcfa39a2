"""Failure detection on the GPU without a fault.

Every wait of the kernels is bounded (2 s of %globaltimer) and raises an abort
word that ends every other wait, so a failure made on the host ends the launch
with an error code in the scratch block, and the context stays usable:

* an input that never arrives: phase 1 polls an LL vector that nothing writes
  (the flag that nothing sets); its wait runs out, the launch ends with
  kErrInputTimeout, and once the scratch block is zeroed the library computes
  correctly again;
* a cache slot outside the cache: the attention phase raises kErrBadInput
  instead of reading or writing past the cache, the engine reports it and
  resets its device state, and the next request decodes exactly as before;
  the batched engine does the same when one of its streams has such a slot;
* a launch on a scratch block that still holds an error (no reset after the
  abort) is refused on the device: nothing is written and nothing advances;
* a program that does not suit the lean kernel, launched with the lean flag,
  aborts at its first unsuitable phase with kErrBadPhase.
"""
import ctypes
import time

import numpy as np
import pytest
import torch

from _native import (F_LL_IN, F_LL_OUT, PH_GEMV, PROGRAM_LEAN, AicasError, AicasPhase, AicasStepState, check, lib,
                     scratch_bytes)
from _ops import device_error
from batch_engine import Qwen3VLBatchDecodeEngine
from engine import Qwen3VLDecodeEngine
from qwen3vl_config import QWEN3VL_2B, synthetic_prompt, synthetic_state

pytestmark = pytest.mark.gpu
K_ERR_INPUT_TIMEOUT = 16


def test_input_that_never_arrives_ends_the_launch_with_a_timeout(cuda_device):
    L = lib()
    nct = L.aicas_num_ctas(cuda_device.index)
    n, k = 8 * nct, 2048
    g = torch.Generator().manual_seed(0)
    w = (torch.randn(n, k, generator=g) * 0.02).half().to(cuda_device)
    x = torch.randn(k, generator=g).half().to(cuda_device)
    out0 = torch.zeros(n, dtype=torch.int32, device=cuda_device)   # LL words phase 0 writes
    never = torch.zeros(k, dtype=torch.int32, device=cuda_device)  # LL words nothing writes
    out1 = torch.zeros(n, dtype=torch.int32, device=cuda_device)
    p0 = AicasPhase()
    p0.kind, p0.flags, p0.n, p0.k = PH_GEMV, F_LL_OUT, n, k
    p0.w, p0.x, p0.out = w.data_ptr(), x.data_ptr(), out0.data_ptr()
    p1 = AicasPhase()
    p1.kind, p1.flags, p1.n, p1.k = PH_GEMV, F_LL_IN | F_LL_OUT, n, k
    p1.w, p1.x, p1.out, p1.x_src = w.data_ptr(), never.data_ptr(), out1.data_ptr(), 0
    arr = (AicasPhase * 2)(p0, p1)
    check(L.aicas_validate_phases(arr, 2), "aicas_validate_phases")
    prog = torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8).to(cuda_device)
    state = torch.zeros(ctypes.sizeof(AicasStepState), dtype=torch.uint8, device=cuda_device)
    scratch = torch.zeros(scratch_bytes(), dtype=torch.uint8, device=cuda_device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    torch.cuda.synchronize(cuda_device)
    t0 = time.perf_counter()
    check(L.aicas_decode_program_f16(ctypes.c_void_p(prog.data_ptr()), 2, ctypes.c_void_p(state.data_ptr()),
                                     ctypes.c_void_p(scratch.data_ptr()), stream), "aicas_decode_program_f16")
    torch.cuda.synchronize(cuda_device)
    elapsed = time.perf_counter() - t0
    assert device_error(scratch) == K_ERR_INPUT_TIMEOUT
    assert 1.5 < elapsed < 20.0, elapsed  # the 2 s wait limit, then a prompt end
    # phase 0 ran normally before the wait: every word of its output carries its epoch (1)
    assert np.all((out0.cpu().numpy().view(np.uint32) >> 16) == 1)

    # a C-ABI call on the aborted scratch block, made without zeroing it, is
    # refused on the device: no output is written and the error stays recorded
    y0 = torch.full((n,), 7.0, dtype=torch.float16, device=cuda_device)
    check(L.aicas_gemv_f16(ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(w.data_ptr()), None,
                           ctypes.c_void_p(y0.data_ptr()), n, k, ctypes.c_void_p(scratch.data_ptr()), stream),
          "aicas_gemv_f16")
    torch.cuda.synchronize(cuda_device)
    assert torch.all(y0 == 7.0)
    assert device_error(scratch) == K_ERR_INPUT_TIMEOUT

    # with the scratch block zeroed again, the library computes correctly
    scratch.zero_()
    import cuda_decode_gemv as cg

    y = cg.nosplit_matvec_half(x.view(1, k), w, None)
    ref = (w.float() @ x.float()).view(1, n)
    assert torch.allclose(y.float(), ref, atol=2e-2, rtol=1e-2)


def test_cache_slot_outside_the_cache_is_reported_not_used(cuda_device):
    shape = QWEN3VL_2B.with_layers(2)
    st = synthetic_state(shape, seed=0)
    eng = Qwen3VLDecodeEngine(st, shape, max_cache_len=64, max_steps=128)
    prompt = synthetic_prompt(20, seed=9).numpy()
    ref = eng.generate(prompt, 8)
    kv = (eng.k_cache.clone(), eng.v_cache.clone())
    start = torch.tensor([int(ref[0]), eng.max_cache_len, 40, 40, 40], dtype=torch.int64)  # slot == cache length
    eng.decode_host(start, 1, graph_steps=1)
    # a further step launched without resetting the device state is refused:
    # the step state, the caches and the recorded error stay as they were
    st_after = eng.state_dev.clone()
    eng.launch(2)
    torch.cuda.synchronize(cuda_device)
    assert torch.equal(eng.state_dev, st_after)
    assert device_error(eng.scratch) == 15
    with pytest.raises(AicasError, match="device error 15"):
        eng.check_error()
    # nothing was written into the cache
    assert torch.equal(eng.k_cache, kv[0]) and torch.equal(eng.v_cache, kv[1])
    again = eng.generate(prompt, 8)
    assert torch.equal(again, ref)


def test_batched_stream_with_a_slot_outside_the_cache_is_reported_not_used(cuda_device):
    shape = QWEN3VL_2B.with_layers(2)
    st = synthetic_state(shape, seed=0)
    eng = Qwen3VLBatchDecodeEngine(st, shape, max_batch=3, max_cache_len=64, max_steps=128)
    prompts = [synthetic_prompt(n, seed=sd).numpy() for n, sd in ((20, 9), (7, 10), (33, 11))]
    ref = eng.generate_batch(prompts, 8)
    kv1 = (eng.k_cache[:, 1].clone(), eng.v_cache[:, 1].clone())
    start = torch.tensor([[int(ref[b][0]), len(prompts[b])] + [len(prompts[b])] * 3 for b in range(3)],
                         dtype=torch.int64)
    start[1, 1] = eng.max_cache_len  # stream 1: slot == cache length
    eng.decode_host(start, 1, graph_steps=1)
    with pytest.raises(AicasError, match="device error 15"):
        eng.check_error()
    # nothing was written into stream 1's cache
    assert torch.equal(eng.k_cache[:, 1], kv1[0]) and torch.equal(eng.v_cache[:, 1], kv1[1])
    again = eng.generate_batch(prompts, 8)
    for b in range(3):
        assert torch.equal(again[b], ref[b]), b


def test_lean_flag_on_a_program_that_does_not_qualify_aborts(cuda_device):
    L = lib()
    nct = L.aicas_num_ctas(cuda_device.index)
    n, k = 256, 1024  # part of a 2048-column chunk: not a lean phase
    g = torch.Generator().manual_seed(1)
    w = (torch.randn(n, k, generator=g) * 0.02).half().to(cuda_device)
    x = torch.randn(k, generator=g).half().to(cuda_device)
    y = torch.zeros(n, dtype=torch.float16, device=cuda_device)
    p0 = AicasPhase()
    p0.kind, p0.n, p0.k = PH_GEMV, n, k
    p0.w, p0.x, p0.out = w.data_ptr(), x.data_ptr(), y.data_ptr()
    arr = (AicasPhase * 1)(p0)
    check(L.aicas_validate_phases(arr, 1), "aicas_validate_phases")
    assert L.aicas_lean_program_ok(arr, 1, nct) != 0
    prog = torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8).to(cuda_device)
    state = torch.zeros(ctypes.sizeof(AicasStepState), dtype=torch.uint8, device=cuda_device)
    scratch = torch.zeros(scratch_bytes(), dtype=torch.uint8, device=cuda_device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)

    def launch(flags):
        check(L.aicas_decode_program_ex_f16(ctypes.c_void_p(prog.data_ptr()), 1, ctypes.c_void_p(state.data_ptr()),
                                            ctypes.c_void_p(scratch.data_ptr()), None, flags, stream),
              "aicas_decode_program_ex_f16")
        torch.cuda.synchronize(cuda_device)

    t0 = time.perf_counter()
    launch(PROGRAM_LEAN)
    assert time.perf_counter() - t0 < 5.0  # the abort ends every wait at once
    assert device_error(scratch) == 14
    scratch.zero_()
    launch(0)
    assert device_error(scratch) == 0
    assert torch.allclose(y.float(), w.float() @ x.float(), atol=2e-2, rtol=1e-2)
