"""Pin the CPU oracle to golden vectors produced by the reference itself
(`tests/golden/make_golden.py`: the reference's `GreedyDecodeEngine`,
`_decode_one_token_eager` and `_hf_repeat_kv_attention` on HF transformers
5.5.0, fp32 CPU)."""
from pathlib import Path

import numpy as np
import pytest

from oracle.qwen3vl_oracle import Qwen3VLOracle, attention_reference
from qwen3vl_config import QWEN3VL_2B, synthetic_state

GOLDEN = Path(__file__).resolve().parent / "golden"
FP32_ATOL = 1e-4  # fp32 check path vs the reference's fp32 CPU path


@pytest.fixture(scope="module")
def state2():
    return synthetic_state(QWEN3VL_2B.with_layers(2), seed=0)


def _check_logits(logits, g):
    assert np.abs(logits[:, g["sample_idx"]] - g["sample_logits"]).max() <= FP32_ATOL
    top = np.take_along_axis(logits, g["top_idx"], axis=-1)
    assert np.abs(top - g["top_val"]).max() <= FP32_ATOL


def test_greedy_text_matches_reference_engine(state2):
    g = np.load(GOLDEN / "greedy_text.npz")
    o = Qwen3VLOracle(state2, 2, mode="fp32", max_cache_len=128)
    toks, logits = o.greedy(g["prompt"], len(g["tokens"]))
    np.testing.assert_array_equal(toks, g["tokens"])
    _check_logits(logits, g)


def test_vision_grid_mrope_matches_reference(state2):
    g = np.load(GOLDEN / "vision_grid.npz")
    o = Qwen3VLOracle(state2, 2, mode="fp32", max_cache_len=320)
    toks, logits = o.greedy(g["prompt"], len(g["tokens"]), pos3_prompt=g["pos3"], rope_delta=int(g["rope_delta"]))
    np.testing.assert_array_equal(toks, g["tokens"])
    _check_logits(logits, g)


def test_interleaved_mrope_tables():
    g = np.load(GOLDEN / "rope.npz")
    o = Qwen3VLOracle({"embed_tokens.weight": np.zeros((1, 1)), "norm.weight": np.zeros(1)}, 0, mode="fp32",
                      max_cache_len=1)
    np.testing.assert_allclose(o.inv_freq, g["inv_freq"], rtol=1e-6, atol=0)
    cos, sin = o.mrope_cos_sin(g["pos3"])
    np.testing.assert_allclose(cos, g["cos"], atol=1e-5)
    np.testing.assert_allclose(sin, g["sin"], atol=1e-5)


@pytest.mark.parametrize("L", [128, 777])
def test_attention_matches_hf_repeat_kv(L):
    import torch

    g = np.load(GOLDEN / "attention.npz")
    gen = torch.Generator().manual_seed(500 + L)
    q = torch.randn((1, 16, 1, 128), generator=gen)
    k = torch.randn((1, 8, L, 128), generator=gen)
    v = torch.randn((1, 8, L, 128), generator=gen)
    out = attention_reference(q.reshape(16, 128).numpy(), k[0].numpy(), v[0].numpy(), L, 128 ** -0.5)
    np.testing.assert_allclose(out, g[f"out_{L}"], atol=1e-5)


def test_oracle_fp16_mode_tracks_fp32(state2):
    """The fp16-rounding checker stays within the fp16 tolerance of the
    reference's fp32 trajectory on the golden prompt (same tokens)."""
    g = np.load(GOLDEN / "greedy_text.npz")
    o = Qwen3VLOracle(state2, 2, mode="fp16", max_cache_len=128)
    toks, logits = o.greedy(g["prompt"], len(g["tokens"]))
    np.testing.assert_array_equal(toks, g["tokens"])
    assert np.abs(logits[:, g["sample_idx"]] - g["sample_logits"]).max() <= 2e-2


class _ChunkedMropeOracle(Qwen3VLOracle):
    """Planted mistake: chunked [TTT..HHH..WWW] MRoPE (Qwen2-VL layout)
    instead of Qwen3-VL's interleaved one."""

    def mrope_cos_sin(self, pos3):
        pos3 = np.asarray(pos3, dtype=np.int64).reshape(3, -1)
        freqs = self.inv_freq[None, None, :] * pos3.astype(np.float32)[:, :, None]
        a, b, _ = self.mrope_section
        out = np.concatenate([freqs[0][:, :a], freqs[1][:, a:a + b], freqs[2][:, a + b:]], axis=-1)
        emb = np.concatenate([out, out], axis=-1)
        return self._round(np.cos(emb)), self._round(np.sin(emb))


def test_planted_mistake_is_caught(state2):
    """The golden pin must reject an oracle with the wrong MRoPE layout."""
    g = np.load(GOLDEN / "vision_grid.npz")
    o = _ChunkedMropeOracle(state2, 2, mode="fp32", max_cache_len=320)
    _, logits = o.greedy(g["prompt"], 2, pos3_prompt=g["pos3"], rope_delta=int(g["rope_delta"]))
    assert np.abs(logits[:, g["sample_idx"]] - g["sample_logits"][:2]).max() > 1e-3
