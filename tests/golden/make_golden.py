"""Generate the golden vectors that pin the CPU oracle to the reference.

Run in the build container (where the read-only reference checkout and HF
transformers 5.5.0 are importable):

    python tests/golden/make_golden.py --reference <path to reference checkout>

It writes small `.npz` fixtures next to this file; the tests read only those
fixtures (the reference is never needed at test time).  Inputs are NOT stored:
weights and prompts are regenerated from their seeds by
`qwen3vl_config.synthetic_state` / `synthetic_prompt` (torch CPU generators are
deterministic for a given torch build).

Cases
-----
greedy_text.npz   BASELINE config 1: 2-layer fp32 model, 64-token prompt, the
                  reference's own `GreedyDecodeEngine.generate`
                  (`evaluation_wrapper.py:149-315`, ENABLE_CUDAGRAPH=0 so the
                  eager step `_decode_one_token_eager` `:513-539` runs), 33 new
                  tokens (1 from prefill + 32 decode steps).  Logits of every
                  step are captured by a hook on `lm_head`; stored: ids, top-32
                  (value, index) per step and the logits at 2048 fixed indices.
vision_grid.npz   2-layer fp32 model, 300-token prefix whose slots 16..271 are
                  a 16x16 image grid with 3-axis MRoPE positions (HF forward
                  with explicit `position_ids`), then 12 decode steps through
                  the reference's `_decode_one_token_eager` with
                  rope_deltas = -240.
rope.npz          HF `Qwen3VLTextRotaryEmbedding` inv_freq and fp32 cos/sin for
                  the grid positions (pins the interleaved-MRoPE mapping).
attention.npz     `_hf_repeat_kv_attention` (`bench_decode_attention.py:241-261`)
                  on seeded fp32 q [1,16,1,128], K/V [1,8,L,128], L in {128, 777}.
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO / "aicasgc-2026_b200"))

from qwen3vl_config import (  # noqa: E402
    QWEN3VL_2B, hf_model, synthetic_prompt, vision_grid_positions,
)

N_LAYERS = 2
SAMPLE_IDX_SEED = 99
N_SAMPLE = 2048
TOPK = 32


def sample_indices(vocab: int) -> np.ndarray:
    rng = np.random.default_rng(SAMPLE_IDX_SEED)
    return np.sort(rng.choice(vocab, size=N_SAMPLE, replace=False)).astype(np.int64)


def summarize(logits_rows: np.ndarray):
    idx = sample_indices(logits_rows.shape[-1])
    top_i = np.argsort(-logits_rows, axis=-1, kind="stable")[:, :TOPK]
    top_v = np.take_along_axis(logits_rows, top_i, axis=-1)
    return dict(sample_idx=idx, sample_logits=logits_rows[:, idx].astype(np.float32),
                top_idx=top_i.astype(np.int64), top_val=top_v.astype(np.float32))


def build_hf_model(n_layers: int):
    return hf_model(QWEN3VL_2B.with_layers(n_layers), seed=0)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    args = ap.parse_args()

    os.environ["ENABLE_CUDAGRAPH"] = "0"
    sys.path.insert(0, args.reference)
    import torch
    import evaluation_wrapper as ew  # the reference's engine
    import bench_decode_attention as bda  # the reference's attention oracle
    from transformers.cache_utils import StaticCache

    torch.set_num_threads(os.cpu_count())
    model = build_hf_model(N_LAYERS)
    captured = []
    model.lm_head.register_forward_hook(
        lambda _m, _i, out: captured.append(out.detach()[0, -1].float().numpy().copy()))

    # ---- case 1: greedy text decode through the reference engine ----------
    prompt = synthetic_prompt(64, seed=1234).view(1, -1)
    engine = ew.GreedyDecodeEngine(model, max_tokens_threshold=128)
    with torch.no_grad():
        out = engine.generate(prompt, attention_mask=torch.ones_like(prompt),
                              max_new_tokens=33, do_sample=False)
    gen = out[0, 64:].numpy().astype(np.int64)
    rows = np.stack(captured)
    assert rows.shape[0] == 33, rows.shape
    np.savez_compressed(HERE / "greedy_text.npz", prompt=prompt[0].numpy(), tokens=gen,
                        n_layers=N_LAYERS, **summarize(rows))
    print("greedy_text tokens", gen.tolist())

    # ---- case 2: vision-grid MRoPE prefix + decode -------------------------
    captured.clear()
    P = 300
    pos3, rope_delta = vision_grid_positions(P)
    assert rope_delta == -240
    vprompt = synthetic_prompt(P, seed=4321).view(1, -1)
    cache = StaticCache(config=model.config, max_cache_len=P + 16)
    with torch.no_grad():
        o = model(input_ids=vprompt, attention_mask=torch.ones_like(vprompt),
                  position_ids=pos3.view(3, 1, P), past_key_values=cache, use_cache=True,
                  cache_position=torch.arange(P), logits_to_keep=1)
        nxt = torch.argmax(o.logits[:, -1, :], dim=-1, keepdim=True)
        full_mask = torch.zeros((1, P + 16), dtype=torch.bool)
        full_mask[:, :P] = True
        toks = [int(nxt)]
        rd = torch.tensor([[rope_delta]], dtype=torch.long)
        for step in range(11):
            nxt = engine._decode_one_token_eager(next_tokens=nxt, full_attention_mask=full_mask,
                                                 rope_deltas=rd, static_cache=cache,
                                                 current_position=P + step,
                                                 device=torch.device("cpu"))
            toks.append(int(nxt))
    rows = np.stack(captured)
    assert rows.shape[0] == 12, rows.shape
    np.savez_compressed(HERE / "vision_grid.npz", prompt=vprompt[0].numpy(), pos3=pos3.numpy(),
                        rope_delta=rope_delta, tokens=np.asarray(toks, np.int64),
                        n_layers=N_LAYERS, **summarize(rows))
    print("vision_grid tokens", toks)

    # ---- case 3: rotary tables ---------------------------------------------
    rot = model.model.language_model.rotary_emb
    probe = torch.zeros(1, 1, QWEN3VL_2B.hidden)
    cos, sin = rot(probe, pos3.view(3, 1, P))
    np.savez_compressed(HERE / "rope.npz", inv_freq=rot.inv_freq.numpy(), pos3=pos3.numpy(),
                        cos=cos[0].numpy(), sin=sin[0].numpy())

    # ---- case 4: decode attention op ---------------------------------------
    res = {}
    for L in (128, 777):
        g = torch.Generator().manual_seed(500 + L)
        q = torch.randn((1, 16, 1, 128), generator=g)
        k = torch.randn((1, 8, L, 128), generator=g)
        v = torch.randn((1, 8, L, 128), generator=g)
        o = bda._hf_repeat_kv_attention(q, k, v, None, 128 ** -0.5, 2)
        res[f"out_{L}"] = o.reshape(16, 128).numpy()
    np.savez_compressed(HERE / "attention.npz", **res)
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()
