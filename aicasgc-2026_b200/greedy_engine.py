"""Drop-in for the reference's `GreedyDecodeEngine` (evaluation_wrapper.py:74-315).

Same constructor (`GreedyDecodeEngine(model, max_tokens_threshold)`), same
request check (`is_supported` / `SUPPORTED_KWARGS`, evaluation_wrapper.py:98-127)
and same `generate(input_ids, attention_mask=..., pixel_values=...,
image_grid_thw=..., max_new_tokens=..., eos_token_id=...)` returning
`output_ids [1, prompt + generated]` (the prompt followed by the greedy tokens,
cut after the first end-of-sequence token, which is kept).

What runs where:

* the prompt: a text-only prompt is prefilled by the native one-pass prefill
  (`Qwen3VLDecodeEngine.prefill_prompt`); a prompt with images goes through the
  HF model's own forward (vision tower + text decoder into a `StaticCache`),
  exactly as the reference prefills (evaluation_wrapper.py:214-227), and its
  K/V slots and `rope_deltas` are handed to the decode engine;
* every decode step: the persistent decode kernel (`Qwen3VLDecodeEngine`,
  CUDA graphs, device-side greedy loop and end-of-sequence), with rope
  positions `cache slot + rope_deltas` on all three axes like the reference's
  `_build_decode_position_ids` (evaluation_wrapper.py:507-511).

A request the reference would refuse raises `ValueError` with the reference's
reason; `is_supported` tells in advance.  Beyond the reference's rules this
engine needs the prompt plus the new tokens to fit its cache and an
attention mask of ones (the reference pads nothing either: batch 1).
"""
from __future__ import annotations

import torch

from engine import Qwen3VLDecodeEngine
from qwen3vl_config import Qwen3VLTextShape


class GreedyDecodeEngine:
    SUPPORTED_KWARGS = {
        "input_ids",
        "attention_mask",
        "pixel_values",
        "image_grid_thw",
        "mm_token_type_ids",
        "max_new_tokens",
        "do_sample",
        "temperature",
        "use_cache",
        "eos_token_id",
        "pad_token_id",
    }

    def __init__(self, model, max_tokens_threshold: int, *, max_cache_len: int = 4096, graph_steps: int = 32):
        """`model`: an HF `Qwen3VLForConditionalGeneration` on a CUDA device
        (its text decoder's weights are copied once into the decode engine's
        layout; the model itself is used only to prefill prompts with images)."""
        self._model = model
        self._max_tokens_threshold = int(max_tokens_threshold)
        self._graph_steps = int(graph_steps)
        device = next(model.parameters()).device
        if device.type != "cuda":
            raise ValueError("GreedyDecodeEngine needs the model on a CUDA device")
        text_cfg = model.config.get_text_config(decoder=True)
        self._shape = Qwen3VLTextShape.from_hf_text_config(text_cfg)
        state = model.model.language_model.state_dict()
        self._engine = Qwen3VLDecodeEngine(state, self._shape, max_cache_len=max_cache_len, device=device,
                                           max_steps=max_cache_len + 8)
        self._device = device

    @property
    def decode_engine(self) -> Qwen3VLDecodeEngine:
        return self._engine

    # ------------------------------------------------------------ request check
    def is_supported(self, args, kwargs) -> bool:
        return self._get_support_failure_reason(args, kwargs) is None

    def _get_support_failure_reason(self, args, kwargs) -> str | None:
        if len(args) > 1:
            return f"len(args)={len(args)} > 1"
        unsupported = set(kwargs) - self.SUPPORTED_KWARGS
        if unsupported:
            return f"unsupported kwargs: {sorted(unsupported)}"
        input_ids = args[0] if args else kwargs.get("input_ids")
        if input_ids is None or input_ids.ndim != 2:
            return f"input_ids must be rank-2, got {None if input_ids is None else tuple(input_ids.shape)}"
        if input_ids.shape[0] != 1:
            return f"batch_size must be 1, got {input_ids.shape[0]}"
        attention_mask = kwargs.get("attention_mask")
        if attention_mask is not None:
            if attention_mask.ndim != 2:
                return f"attention_mask must be rank-2, got shape={tuple(attention_mask.shape)}"
            if not bool(attention_mask.bool().all()):
                return "attention_mask with padding is unsupported"
        if kwargs.get("do_sample", False):
            return "do_sample=True is unsupported"
        if not kwargs.get("use_cache", True):
            return "use_cache=False is unsupported"
        max_new_tokens = kwargs.get("max_new_tokens", self._max_tokens_threshold)
        if max_new_tokens is None or max_new_tokens < 1:
            return f"max_new_tokens must be >=1, got {max_new_tokens}"
        if max_new_tokens > self._max_tokens_threshold:
            return f"max_new_tokens={max_new_tokens} exceeds threshold={self._max_tokens_threshold}"
        P = input_ids.shape[1]
        if P < 1 or P + max_new_tokens - 1 > self._engine.max_cache_len:
            return f"prompt {P} + max_new_tokens {max_new_tokens} exceeds the cache ({self._engine.max_cache_len})"
        return None

    def _eos_values(self, kwargs) -> list[int]:
        """The request's end-of-sequence ids: `eos_token_id`, else the model's
        generation config, else its text config (evaluation_wrapper.py:468-510)."""
        eos = kwargs.get("eos_token_id")
        if eos is None:
            gen_cfg = getattr(self._model, "generation_config", None)
            eos = getattr(gen_cfg, "eos_token_id", None) if gen_cfg is not None else None
        if eos is None:
            eos = getattr(self._model.config.get_text_config(decoder=True), "eos_token_id", None)
        if eos is None:
            return []
        if isinstance(eos, torch.Tensor):
            return [int(x) for x in eos.detach().cpu().view(-1).tolist()]
        if isinstance(eos, (list, tuple, set)):
            return [int(x) for x in eos]
        return [int(eos)]

    # ---------------------------------------------------------------- generate
    @torch.no_grad()
    def generate(self, *args, **kwargs) -> torch.Tensor:
        reason = self._get_support_failure_reason(args, kwargs)
        if reason is not None:
            raise ValueError(f"unsupported request: {reason}")
        input_ids = args[0] if args else kwargs["input_ids"]
        max_new_tokens = int(kwargs.get("max_new_tokens", self._max_tokens_threshold))
        eos = self._eos_values(kwargs)
        device_eos = eos[0] if eos else None  # the device stops at this one; the others are cut on the host
        P = input_ids.shape[1]
        eng = self._engine
        prompt = input_ids[0].to(torch.int64)
        if kwargs.get("pixel_values") is None:
            eng.prefill_prompt(prompt.cpu(), None, eos_token_id=device_eos)
        else:
            first, delta = self._hf_prefill(input_ids, kwargs)
            eng.begin_decode(first, P, [P + delta] * 3, device_eos)
        eng.run(max_new_tokens - 1, self._graph_steps)
        toks = eng.collect(P, max_new_tokens)
        if len(eos) > 1:  # cut at the first of any end-of-sequence id (kept)
            hit = [i for i, t in enumerate(toks.tolist()) if t in eos]
            if hit:
                toks = toks[:hit[0] + 1]
        return torch.cat([input_ids, toks.view(1, -1).to(device=input_ids.device, dtype=input_ids.dtype)], 1)

    def _hf_prefill(self, input_ids, kwargs):
        """Prompt with images: the HF model's forward (vision tower + text
        decoder) into a StaticCache, then its K/V slots [0, P) copied into the
        decode engine's cache.  Returns (first token, rope delta)."""
        from transformers.cache_utils import StaticCache

        P = input_ids.shape[1]
        cache = StaticCache(config=self._model.config, max_cache_len=P)
        mask = kwargs.get("attention_mask")
        if mask is None:
            mask = torch.ones_like(input_ids, dtype=torch.bool)
        out = self._model(input_ids=input_ids, attention_mask=mask, pixel_values=kwargs.get("pixel_values"),
                          image_grid_thw=kwargs.get("image_grid_thw"),
                          mm_token_type_ids=kwargs.get("mm_token_type_ids"), past_key_values=cache,
                          use_cache=True, logits_to_keep=1)
        eng = self._engine
        for li, layer in enumerate(cache.layers):
            eng.k_cache[li][:, :, :P].copy_(layer.keys[:, :, :P])
            eng.v_cache[li][:, :, :P].copy_(layer.values[:, :, :P])
        delta = 0 if out.rope_deltas is None else int(out.rope_deltas.view(-1)[0])
        first = int(torch.argmax(out.logits[0, -1]))
        return first, delta
