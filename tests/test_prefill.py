"""The one-pass causal prefill (prefill.py) against the CPU oracle's prefill
on a 2-layer model with a vision-grid prompt (3-axis MRoPE positions): logits
of the last prompt token and every K/V slot it writes.  Runs on the CPU
(torch CPU tensors); the engine runs the same function on CUDA."""
import numpy as np
import torch

from engine import hf_inv_freq
from oracle.qwen3vl_oracle import Qwen3VLOracle
from prefill import layer_weights_from_hf, prefill
from qwen3vl_config import QWEN3VL_2B, synthetic_prompt, synthetic_state, vision_grid_positions


def test_prefill_matches_oracle_prefill():
    shape = QWEN3VL_2B.with_layers(2)
    st = synthetic_state(shape, seed=0, dtype=torch.float16)
    P, Lmax = 48, 64
    tokens = synthetic_prompt(P, seed=11)
    pos3, _ = vision_grid_positions(P)
    inv = hf_inv_freq(shape)
    kc = torch.zeros((2, 1, shape.num_kv_heads, Lmax, shape.head_dim), dtype=torch.float16)
    vc = torch.zeros_like(kc)
    logits = prefill(tokens, pos3, st["embed_tokens.weight"], st["norm.weight"], layer_weights_from_hf(st, 2), kc, vc,
                     num_heads=shape.num_heads, num_kv_heads=shape.num_kv_heads, head_dim=shape.head_dim,
                     eps=shape.rms_eps, inv_freq=inv, mrope_section=shape.mrope_section)
    o = Qwen3VLOracle(st, 2, mode="fp16", max_cache_len=Lmax, inv_freq=inv.numpy())
    ref = o.prefill(tokens.numpy(), pos3.numpy())
    got = logits.numpy()
    assert np.abs(got - ref).max() < 2e-2, np.abs(got - ref).max()
    assert int(np.argmax(got)) == int(np.argmax(ref))
    for li in range(2):
        for cache, ocache in ((kc, o.k_cache), (vc, o.v_cache)):
            a = cache[li, 0, :, :P].float().numpy()
            b = ocache[li, :, :P]
            assert np.abs(a - b).max() <= 2e-2 * max(1.0, np.abs(b).max()), np.abs(a - b).max()
        assert float(kc[li, 0, :, P:].abs().sum()) == 0.0  # nothing written past the prompt


def test_prefill_k_blocked_down_equals_plain_down():
    """The engine stores down_proj K-blocked; both layouts give the same result."""
    shape = QWEN3VL_2B.with_layers(1)
    st = synthetic_state(shape, seed=0, dtype=torch.float16)
    P, Lmax = 16, 32
    tokens = synthetic_prompt(P, seed=12)
    pos3 = torch.arange(P, dtype=torch.int64).expand(3, P)
    inv = hf_inv_freq(shape)
    lw = layer_weights_from_hf(st, 1)
    lwb = [dict(lw[0], down=lw[0]["down"].view(2048, 3, 2048).permute(1, 0, 2).contiguous())]
    outs = []
    for layers in (lw, lwb):
        kc = torch.zeros((1, 1, shape.num_kv_heads, Lmax, shape.head_dim), dtype=torch.float16)
        outs.append(prefill(tokens, pos3, st["embed_tokens.weight"], st["norm.weight"], layers, kc, torch.zeros_like(kc),
                            num_heads=shape.num_heads, num_kv_heads=shape.num_kv_heads, head_dim=shape.head_dim,
                            eps=shape.rms_eps, inv_freq=inv, mrope_section=shape.mrope_section))
    assert np.abs(outs[0].numpy() - outs[1].numpy()).max() < 2e-2
