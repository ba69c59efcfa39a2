"""`optimized_layer` drop-in on the GPU, driven by its real caller: HF's own
Qwen3-VL model (layer loop, rotary embedding, StaticCache, lm_head).

`replace_decoder_layers` swaps the two decoder layers of the 2-layer
synthetic model (fp16, CUDA); HF prefills the prompt through the layers'
HF path, and every single-token step then runs the five drop-in ops (the
B200 kernels) inside HF's forward.  Checks: the reference engine's golden
greedy tokens reproduced exactly (tests/golden/greedy_text.npz, BASELINE
config 1: 64-token prompt, 33 new tokens), every decode step served by the
kernels, and logits within 2e-2 of HF's own fp16 decode of the same tokens
(the unmodified HF layers on the GPU, teacher-forced).
"""
from pathlib import Path

import numpy as np
import pytest
import torch

pytest.importorskip("transformers")

from optimized_layer import replace_decoder_layers  # noqa: E402
from qwen3vl_config import QWEN3VL_2B, hf_model, synthetic_state  # noqa: E402

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
LOGIT_ATOL = 2e-2


@torch.no_grad()
def _greedy(model, prompt, n, forced=None):
    """Prefill `prompt`, then n - 1 single-token steps through `model` with a
    StaticCache; explicit 3-axis text positions.  Returns (tokens, fp32 logits)."""
    from transformers.cache_utils import StaticCache

    dev = next(model.parameters()).device
    P = len(prompt)
    cache = StaticCache(config=model.config, max_cache_len=P + n)
    ids = torch.as_tensor(prompt, dtype=torch.long, device=dev).view(1, P)
    pos = torch.arange(P, device=dev).view(1, 1, P).expand(3, 1, P)
    logits = [model(input_ids=ids, position_ids=pos, past_key_values=cache, use_cache=True,
                    logits_to_keep=1).logits[0, -1].float()]
    toks = [int(logits[-1].argmax())]
    for i in range(n - 1):
        inp = toks[-1] if forced is None else int(forced[i])
        p = torch.full((3, 1, 1), P + i, dtype=torch.long, device=dev)
        out = model(input_ids=torch.tensor([[inp]], device=dev), position_ids=p, past_key_values=cache,
                    use_cache=True)
        logits.append(out.logits[0, -1].float())
        toks.append(int(logits[-1].argmax()))
    return np.asarray(toks, np.int64), torch.stack(logits).cpu().numpy()


def test_replaced_layers_reproduce_reference_tokens_and_hf_logits(cuda_device):
    g = np.load(GOLDEN / "greedy_text.npz")
    n = len(g["tokens"])
    state = synthetic_state(QWEN3VL_2B.with_layers(2), seed=0)
    model = hf_model(QWEN3VL_2B.with_layers(2), state=state).half().to(cuda_device)
    assert replace_decoder_layers(model) == 2
    toks, lg = _greedy(model, g["prompt"], n)
    np.testing.assert_array_equal(toks, g["tokens"])
    layers = model.model.language_model.layers
    assert [m.decode_steps for m in layers] == [n - 1, n - 1]
    del model
    hf = hf_model(QWEN3VL_2B.with_layers(2), state=state).half().to(cuda_device)
    _, hl = _greedy(hf, g["prompt"], n, forced=toks)
    d = np.abs(lg - hl).max(axis=-1)
    print(f"\ndrop-in layers vs HF fp16 decode: max |d logit| per step {np.round(d, 4).tolist()}")
    assert d.max() <= LOGIT_ATOL
