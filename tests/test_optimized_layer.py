"""`optimized_layer` drop-in on the CPU: the HF path of OptimizedDecoderLayer.

On the CPU (and for any input the decode kernels do not take) the layer runs
HF's decoder-layer math over its fused weights, so a model whose layers were
replaced by `replace_decoder_layers` must give HF's own logits: full-sequence
forward, and a StaticCache prefill followed by single-token steps.  A small
text decoder keeps this quick; the decode kernels themselves are tested on the
GPU (tests/test_optimized_layer_gpu.py).
"""
import pytest
import torch

pytest.importorskip("transformers")

from optimized_layer import OptimizedDecoderLayer, replace_decoder_layers  # noqa: E402
from qwen3vl_config import Qwen3VLTextShape, hf_model, synthetic_prompt  # noqa: E402

SMALL = Qwen3VLTextShape(hidden=256, num_heads=4, num_kv_heads=2, head_dim=64, intermediate=512, vocab=1000,
                         num_layers=2, mrope_section=(8, 12, 12))


@pytest.fixture(scope="module")
def models():
    torch.set_grad_enabled(False)
    ref = hf_model(SMALL)
    opt = hf_model(SMALL)
    assert replace_decoder_layers(opt) == 2
    assert replace_decoder_layers(opt) == 0  # already replaced
    assert all(isinstance(m, OptimizedDecoderLayer) for m in opt.model.language_model.layers)
    return ref, opt


def test_replaced_model_matches_hf_full_forward(models):
    ref, opt = models
    ids = synthetic_prompt(12, seed=3, vocab_limit=SMALL.vocab).view(1, -1)
    a = ref(input_ids=ids).logits
    b = opt(input_ids=ids).logits
    torch.testing.assert_close(b, a, atol=1e-4, rtol=1e-4)


def test_replaced_model_matches_hf_with_static_cache(models):
    from transformers.cache_utils import StaticCache

    ref, opt = models
    P, n = 10, 4
    ids = synthetic_prompt(P, seed=4, vocab_limit=SMALL.vocab).view(1, -1)
    outs = []
    for m in (ref, opt):
        cache = StaticCache(config=m.config, max_cache_len=P + n)
        pos = torch.arange(P).view(1, 1, P).expand(3, 1, P)
        lg = [m(input_ids=ids, position_ids=pos, past_key_values=cache, use_cache=True).logits[0, -1]]
        tok = int(lg[-1].argmax())
        for i in range(n - 1):
            p = torch.full((3, 1, 1), P + i, dtype=torch.long)
            lg.append(m(input_ids=torch.tensor([[tok]]), position_ids=p, past_key_values=cache,
                        use_cache=True).logits[0, -1])
            tok = int(lg[-1].argmax())
        outs.append(torch.stack(lg))
        assert int(cache.layers[0].cumulative_length) == P + n - 1
    torch.testing.assert_close(outs[1], outs[0], atol=1e-4, rtol=1e-4)
    # the CPU path never reaches the decode kernels
    assert all(m.decode_steps == 0 for m in models[1].model.language_model.layers)
