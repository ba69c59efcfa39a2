"""The native one-pass prefill on the GPU (prefill_native: the library's
prefill kernels between fp16 GEMMs).

* The causal flash-attention kernel against fp32 causal attention (torch on
  the GPU, the oracle's formula) for prompt lengths around the 64-query and
  64-key tile edges, GQA 2:1.  Its only extra rounding point is P rounded to
  fp16 for the P V product, so outputs agree to a few fp16 ulps.
* The whole prefill against the CPU oracle's prefill (2 layers, vision-grid
  positions): logits of the last prompt token within 2e-2 with the same
  argmax, and every K/V slot it writes.
"""
import ctypes

import numpy as np
import pytest
import torch

import _native
from engine import hf_inv_freq
from oracle.qwen3vl_oracle import Qwen3VLOracle
from prefill import layer_weights_from_hf, prefill
from qwen3vl_config import QWEN3VL_2B, synthetic_prompt, synthetic_state, vision_grid_positions

pytestmark = pytest.mark.gpu


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _causal_attention_ref(q, k, v, P, start=0):
    """fp32 causal GQA attention: q [P, Hq, D] at cache slots start .., k/v
    [Hkv, >= start + P, D]."""
    hq, hkv = q.shape[1], k.shape[0]
    L = start + P
    qf = q.float().transpose(0, 1)                                            # [Hq, P, D]
    kf = k[:, :L].float().repeat_interleave(hq // hkv, 0)                     # [Hq, L, D]
    vf = v[:, :L].float().repeat_interleave(hq // hkv, 0)
    s = (qf @ kf.transpose(1, 2)) * q.shape[-1] ** -0.5
    qi = torch.arange(P, device=q.device).view(-1, 1) + start
    s = s.masked_fill(torch.arange(L, device=q.device).view(1, -1) > qi, float("-inf"))
    return (torch.softmax(s, -1) @ vf).transpose(0, 1)                         # [P, Hq, D]


@pytest.mark.parametrize("P,start", [(1, 0), (5, 0), (63, 0), (64, 0), (65, 0), (127, 0), (128, 0), (129, 0),
                                     (300, 0), (1024, 0), (100, 200), (1, 511), (257, 3)])
def test_prefill_attention_kernel(cuda_device, P, start):
    """The tcgen05 attention through its HF-layout entry point: queries at
    cache slots start .. start + P - 1 over slots [0, start + t] (a
    workspace full of NaN bit patterns: every byte the kernel reads is
    written first)."""
    L = _native.lib()
    g = torch.Generator(device=cuda_device).manual_seed(100 + P + start)
    lmax = start + P + 37
    q = torch.randn((P, 16, 128), generator=g, device=cuda_device).half()
    k = torch.randn((8, lmax, 128), generator=g, device=cuda_device).half()
    v = torch.randn((8, lmax, 128), generator=g, device=cuda_device).half()
    out = torch.full((P, 16, 128), float("nan"), dtype=torch.float16, device=cuda_device)
    ws = torch.full((L.aicas_prefill_attention_workspace_bytes(P, start, 16, 8),), 0xFF, dtype=torch.uint8,
                    device=cuda_device)
    rc = L.aicas_prefill_attention_f16(_p(q), _p(k), _p(v), _p(out), P, start, 16, 8, lmax, 128 ** -0.5, _p(ws),
                                       ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _native.check(rc, "aicas_prefill_attention_f16")
    ref = _causal_attention_ref(q, k, v, P, start)
    err = (out.float() - ref).abs().max().item()
    assert err <= 4e-3, err
    assert L.aicas_prefill_attention_timeouts() == 0


def test_prefill_native_matches_oracle_prefill(cuda_device):
    shape = QWEN3VL_2B.with_layers(2)
    st = synthetic_state(shape, seed=0, dtype=torch.float16)
    P, Lmax = 300, 320
    tokens = synthetic_prompt(P, seed=11)
    pos3, _ = vision_grid_positions(P)
    inv = hf_inv_freq(shape)
    layers = [{k: v.to(cuda_device) for k, v in lw.items()} for lw in layer_weights_from_hf(st, 2)]
    kc = torch.zeros((2, 1, shape.num_kv_heads, Lmax, shape.head_dim), dtype=torch.float16, device=cuda_device)
    vc = torch.zeros_like(kc)
    logits = prefill(tokens.to(cuda_device), pos3.to(cuda_device), st["embed_tokens.weight"].to(cuda_device),
                     st["norm.weight"].to(cuda_device), layers, kc, vc, num_heads=shape.num_heads,
                     num_kv_heads=shape.num_kv_heads, head_dim=shape.head_dim, eps=shape.rms_eps, inv_freq=inv,
                     mrope_section=shape.mrope_section)
    o = Qwen3VLOracle(st, 2, mode="fp16", max_cache_len=Lmax, inv_freq=inv.numpy())
    ref = o.prefill(tokens.numpy(), pos3.numpy())
    got = logits.cpu().numpy()
    assert np.abs(got - ref).max() < 2e-2, np.abs(got - ref).max()
    assert int(np.argmax(got)) == int(np.argmax(ref))
    for li in range(2):
        for cache, ocache in ((kc, o.k_cache), (vc, o.v_cache)):
            a = cache[li, 0, :, :P].float().cpu().numpy()
            b = ocache[li, :, :P]
            assert np.abs(a - b).max() <= 2e-2 * max(1.0, np.abs(b).max()), np.abs(a - b).max()
        assert float(kc[li, 0, :, P:].abs().sum()) == 0.0  # nothing written past the prompt
