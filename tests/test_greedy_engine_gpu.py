"""The `GreedyDecodeEngine` drop-in (greedy_engine.py) on the GPU, against
the HF model's own fp16 greedy loop (prefill into a StaticCache, then one
forward per token with rope positions cache slot + rope_deltas), 2 layers:

* a text-only prompt (native one-pass prefill, then the decode kernel);
* a prompt with an image (HF forward through the vision tower for the
  prefill, its K/V and rope_deltas handed to the decode kernel);
* an end-of-sequence id cuts the output after its first occurrence.

Tokens must agree until the HF logits' top two are within 1e-2 of each other
(fp16 sums in a different order may part there)."""
import numpy as np
import pytest
import torch

from greedy_engine import GreedyDecodeEngine
from qwen3vl_config import QWEN3VL_2B, hf_model, synthetic_prompt, synthetic_state

pytestmark = pytest.mark.gpu
TIE = 1e-2


@pytest.fixture(scope="module")
def model(cuda_device):
    shape = QWEN3VL_2B.with_layers(2)
    m = hf_model(shape, state=synthetic_state(shape, seed=0)).half().to(cuda_device)
    return m


def _hf_greedy(model, input_ids, n, **extra):
    from transformers.cache_utils import StaticCache

    P = input_ids.shape[1]
    dev = input_ids.device
    cache = StaticCache(config=model.config, max_cache_len=P + n)
    with torch.no_grad():
        out = model(input_ids=input_ids, attention_mask=torch.ones_like(input_ids), past_key_values=cache,
                    use_cache=True, logits_to_keep=1, **extra)
        delta = 0 if out.rope_deltas is None else int(out.rope_deltas.view(-1)[0])
        logits = [out.logits[0, -1].float()]
        toks = [int(torch.argmax(logits[-1]))]
        for i in range(1, n):
            pos = P + i - 1
            out = model(input_ids=torch.tensor([[toks[-1]]], device=dev),
                        position_ids=torch.full((3, 1, 1), pos + delta, dtype=torch.long, device=dev),
                        cache_position=torch.tensor([pos], device=dev), past_key_values=cache, use_cache=True)
            logits.append(out.logits[0, -1].float())
            toks.append(int(torch.argmax(logits[-1])))
    return toks, torch.stack(logits).cpu().numpy()


def _agree_until_tie(ours, ref, ref_logits):
    srt = np.sort(ref_logits, axis=-1)
    for i, (a, b) in enumerate(zip(ours, ref)):
        if a != b:
            assert srt[i, -1] - srt[i, -2] <= TIE, f"step {i}: {a} vs {b}"
            return i
    return len(ref)


def test_text_prompt_matches_hf_greedy(cuda_device, model):
    eng = GreedyDecodeEngine(model, max_tokens_threshold=32, max_cache_len=256)
    ids = synthetic_prompt(40, seed=77).view(1, -1).to(cuda_device)
    n = 20
    out = eng.generate(ids, attention_mask=torch.ones_like(ids), max_new_tokens=n, do_sample=False)
    assert out.shape == (1, 40 + n) and torch.equal(out[:, :40], ids)
    ref, rl = _hf_greedy(model, ids, n)
    assert _agree_until_tie(out[0, 40:].tolist(), ref, rl) >= 8


def test_image_prompt_matches_hf_greedy(cuda_device, model):
    cfg = model.config
    v = cfg.vision_config
    eng = GreedyDecodeEngine(model, max_tokens_threshold=32, max_cache_len=256)
    grid = torch.tensor([[1, 8, 8]], device=cuda_device)
    n_img = 64 // (v.spatial_merge_size ** 2)
    g = torch.Generator().manual_seed(5)
    pre, post = synthetic_prompt(12, seed=11), synthetic_prompt(10, seed=12)
    ids = torch.cat([pre, torch.tensor([cfg.vision_start_token_id]), torch.full((n_img,), cfg.image_token_id),
                     torch.tensor([cfg.vision_end_token_id]), post]).view(1, -1).to(cuda_device)
    mm = (ids == cfg.image_token_id).to(torch.int32)
    pix = torch.randn(64, v.in_channels * v.temporal_patch_size * v.patch_size ** 2, generator=g).half().to(cuda_device)
    extra = dict(pixel_values=pix, image_grid_thw=grid, mm_token_type_ids=mm)
    n = 16
    out = eng.generate(ids, attention_mask=torch.ones_like(ids), max_new_tokens=n, **extra)
    P = ids.shape[1]
    assert out.shape == (1, P + n) and torch.equal(out[:, :P], ids)
    ref, rl = _hf_greedy(model, ids, n, **extra)
    assert _agree_until_tie(out[0, P:].tolist(), ref, rl) >= 8


def test_end_of_sequence_cuts_the_output(cuda_device, model):
    eng = GreedyDecodeEngine(model, max_tokens_threshold=32, max_cache_len=256)
    ids = synthetic_prompt(30, seed=91).view(1, -1).to(cuda_device)
    full = eng.generate(ids, max_new_tokens=24)[0, 30:].tolist()
    k = next((i for i in range(3, 24) if full[i] not in full[:i]), None)
    if k is None:
        pytest.skip("no fresh token to use as end of sequence")
    cut = eng.generate(ids, max_new_tokens=24, eos_token_id=full[k])[0, 30:].tolist()
    assert cut == full[:k + 1]
    # several ids: the first occurrence of any of them ends the output
    cut2 = eng.generate(ids, max_new_tokens=24, eos_token_id=[999999, full[k]])[0, 30:].tolist()
    assert cut2 == full[:k + 1]
    with pytest.raises(ValueError, match="do_sample"):
        eng.generate(ids, max_new_tokens=4, do_sample=True)
