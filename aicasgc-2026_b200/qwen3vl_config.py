"""Qwen3-VL-2B text-decoder shape constants and the seeded synthetic weights.

The shapes are those of Qwen3-VL-2B-Instruct's text decoder (the model the
reference accelerates, `evaluation_wrapper.py:1109-1114` loads it with
`AutoModelForImageTextToText.from_pretrained`).  The real checkpoint is not
available, so every test and benchmark uses seeded random weights:

* linear and embedding weights ~ N(0, 0.02) (HF's `initializer_range`),
* RMSNorm weights = 1 + N(0, 0.02) (HF initialises them to 1; the small
  perturbation makes the norm-weight multiply observable in parity tests).

Each block of 2048 rows of each tensor has its own `torch.Generator` seeded
from (seed, layer, slot, block), so a 2-layer model's layers equal the first
two layers of the 28-layer model and blocks can be generated in any order on
any number of threads.  Generation runs on the CPU so the values are identical
on every machine with the same torch build.

This module imports torch only inside functions: the oracle tests import the
constants without needing CUDA.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Qwen3VLTextShape:
    hidden: int = 2048
    num_heads: int = 16
    num_kv_heads: int = 8
    head_dim: int = 128
    intermediate: int = 6144
    vocab: int = 151936
    num_layers: int = 28
    rms_eps: float = 1e-6
    rope_theta: float = 5_000_000.0
    mrope_section: tuple = (24, 20, 20)

    @property
    def q_size(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_kv_heads * self.head_dim

    @property
    def qkv_rows(self) -> int:
        return self.q_size + 2 * self.kv_size

    @property
    def groups(self) -> int:
        return self.num_heads // self.num_kv_heads

    def with_layers(self, n: int) -> "Qwen3VLTextShape":
        return Qwen3VLTextShape(**{**self.__dict__, "num_layers": n})

    @staticmethod
    def from_hf_text_config(cfg) -> "Qwen3VLTextShape":
        """The shape of an HF Qwen3-VL text config (`config.get_text_config()`)."""
        rope = getattr(cfg, "rope_parameters", None) or getattr(cfg, "rope_scaling", None) or {}
        theta = rope.get("rope_theta", getattr(cfg, "rope_theta", 5_000_000.0))
        return Qwen3VLTextShape(
            hidden=cfg.hidden_size, num_heads=cfg.num_attention_heads, num_kv_heads=cfg.num_key_value_heads,
            head_dim=getattr(cfg, "head_dim", cfg.hidden_size // cfg.num_attention_heads),
            intermediate=cfg.intermediate_size, vocab=cfg.vocab_size, num_layers=cfg.num_hidden_layers,
            rms_eps=float(cfg.rms_norm_eps), rope_theta=float(theta),
            mrope_section=tuple(rope.get("mrope_section", (24, 20, 20))))

    def weight_bytes_per_step(self) -> int:
        """Algorithmic fp16 weight bytes one decode step must read.

        Per layer: fused QKV [4096x2048], o_proj [2048x2048], gate_up
        [12288x2048], down [2048x6144] plus four norm vectors; then the final
        norm, one embedding row and the tied lm_head [vocab x 2048].
        """
        h, i = self.hidden, self.intermediate
        per_layer = 2 * (self.qkv_rows * h + h * self.q_size + 2 * i * h + h * i)
        norms = 2 * (2 * h + 2 * self.head_dim)
        return self.num_layers * (per_layer + norms) + 2 * h + 2 * h + 2 * self.vocab * h

    def kv_bytes_per_position(self) -> int:
        """K+V bytes of one cached position over all layers (fp16)."""
        return self.num_layers * 2 * self.kv_size * 2


QWEN3VL_2B = Qwen3VLTextShape()

# Slot numbers inside one layer for the per-tensor seeds.
_LAYER_SLOTS = (
    "input_layernorm",
    "q_proj",
    "k_proj",
    "v_proj",
    "o_proj",
    "q_norm",
    "k_norm",
    "post_attention_layernorm",
    "gate_proj",
    "up_proj",
    "down_proj",
)


def _tensor_seed(seed: int, layer: int, slot: int, block: int) -> int:
    # layer -1 holds the model-level tensors (embedding, final norm).
    return (seed * 1_000_003 + (layer + 1) * 1009 + slot * 97 + block) & 0x7FFFFFFFFFFF


# Rows per independently seeded block of a 2-D tensor (lets generation run on
# all host cores while staying independent of thread count and order).
_BLOCK_ROWS = 2048


def layer_tensor_shapes(shape: Qwen3VLTextShape) -> dict:
    h, d = shape.hidden, shape.head_dim
    return {
        "input_layernorm": (h,),
        "q_proj": (shape.q_size, h),
        "k_proj": (shape.kv_size, h),
        "v_proj": (shape.kv_size, h),
        "o_proj": (h, shape.q_size),
        "q_norm": (d,),
        "k_norm": (d,),
        "post_attention_layernorm": (h,),
        "gate_proj": (shape.intermediate, h),
        "up_proj": (shape.intermediate, h),
        "down_proj": (h, shape.intermediate),
    }


def _tensor_meta(shape: Qwen3VLTextShape, layer: int, name: str):
    if layer < 0:
        slot = {"embed_tokens": 0, "norm": 1}[name]
        dims = {"embed_tokens": (shape.vocab, shape.hidden), "norm": (shape.hidden,)}[name]
    else:
        slot = _LAYER_SLOTS.index(name)
        dims = layer_tensor_shapes(shape)[name]
    return slot, dims


def _fill_block(out, seed: int, layer: int, slot: int, block: int, is_norm: bool):
    import torch

    g = torch.Generator(device="cpu")
    g.manual_seed(_tensor_seed(seed, layer, slot, block))
    rows = out[block * _BLOCK_ROWS:(block + 1) * _BLOCK_ROWS] if out.dim() == 2 else out
    t = torch.randn(rows.shape, generator=g, dtype=torch.float32).mul_(0.02)
    if is_norm:  # RMSNorm weight
        t.add_(1.0)
    rows.copy_(t)


def synthetic_tensor(shape: Qwen3VLTextShape, seed: int, layer: int, name: str, dtype=None):
    """One seeded CPU tensor of the synthetic model (see module doc)."""
    import torch

    slot, dims = _tensor_meta(shape, layer, name)
    out = torch.empty(dims, dtype=dtype or torch.float32)
    nblk = 1 if len(dims) == 1 else -(-dims[0] // _BLOCK_ROWS)
    for b in range(nblk):
        _fill_block(out, seed, layer, slot, b, len(dims) == 1)
    return out


def _hf_key(li: int, name: str) -> str:
    if name in ("q_proj", "k_proj", "v_proj", "o_proj", "q_norm", "k_norm"):
        return f"layers.{li}.self_attn.{name}.weight"
    if name in ("gate_proj", "up_proj", "down_proj"):
        return f"layers.{li}.mlp.{name}.weight"
    return f"layers.{li}.{name}.weight"


def synthetic_state(shape: Qwen3VLTextShape, seed: int = 0, dtype=None, threads: int | None = None) -> dict:
    """All tensors of the synthetic text decoder, keyed like HF's state dict
    below `model.language_model.` (`embed_tokens.weight`,
    `layers.{i}.self_attn.q_proj.weight`, ..., `norm.weight`).  Blocks are
    generated on a thread pool; values do not depend on the thread count."""
    import os
    from concurrent.futures import ThreadPoolExecutor

    import torch

    specs = [("embed_tokens.weight", -1, "embed_tokens")]
    for li in range(shape.num_layers):
        specs += [(_hf_key(li, name), li, name) for name in _LAYER_SLOTS]
    specs.append(("norm.weight", -1, "norm"))
    out, jobs = {}, []
    for key, li, name in specs:
        slot, dims = _tensor_meta(shape, li, name)
        t = torch.empty(dims, dtype=dtype or torch.float32)
        out[key] = t
        nblk = 1 if len(dims) == 1 else -(-dims[0] // _BLOCK_ROWS)
        jobs += [(t, li, slot, b, len(dims) == 1) for b in range(nblk)]
    with ThreadPoolExecutor(threads or os.cpu_count() or 1) as ex:
        list(ex.map(lambda j: _fill_block(j[0], seed, j[1], j[2], j[3], j[4]), jobs))
    return out


def synthetic_prompt(n: int, seed: int = 1234, vocab_limit: int = 151643):
    """Prompt token ids drawn uniformly from [0, 151643): below Qwen's special
    and vision token ids, so a text-only prompt never enters multimodal code."""
    import torch

    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    return torch.randint(0, vocab_limit, (n,), generator=g, dtype=torch.int64)


def vision_grid_positions(prefix_len: int, grid_start: int = 16, grid_h: int = 16, grid_w: int = 16):
    """3-axis MRoPE positions (t, h, w) of a synthetic prefix with one image.

    Tokens [grid_start, grid_start + grid_h*grid_w) are an image-placeholder
    grid: t = grid_start, h = grid_start + row, w = grid_start + col (the
    layout HF's `get_vision_position_ids` gives one image with a single
    temporal patch).  Text before the grid has t = h = w = index; text after
    it continues at max(grid position) + 1.  Returns (positions [3, n] int64,
    rope_delta) where rope_delta is the offset a decode step adds to its cache
    position on all three axes (the reference's `_build_decode_position_ids`,
    `evaluation_wrapper.py:507-511`).
    """
    import torch

    pos = torch.empty((3, prefix_len), dtype=torch.int64)
    n_grid = grid_h * grid_w
    end = grid_start + n_grid
    for i in range(min(prefix_len, grid_start)):
        pos[:, i] = i
    for j in range(max(0, min(prefix_len, end) - grid_start)):
        r, c = divmod(j, grid_w)
        pos[0, grid_start + j] = grid_start
        pos[1, grid_start + j] = grid_start + r
        pos[2, grid_start + j] = grid_start + c
    next_text = grid_start + max(grid_h, grid_w)
    for i in range(end, prefix_len):
        pos[:, i] = next_text + (i - end)
    rope_delta = next_text - end
    return pos, rope_delta


def hf_model(shape: Qwen3VLTextShape, seed: int = 0, state: dict | None = None):
    """An HF `Qwen3VLForConditionalGeneration` (transformers 5.x) with the
    text decoder of `shape` and the seeded synthetic weights (`state`, or
    `synthetic_state(shape, seed)`), tied lm_head, SDPA attention, a minimal
    vision tower (unused by text prompts), fp32 on the CPU, in eval mode.
    This is the model the reference's engine runs (`evaluation_wrapper.py:
    1109-1114` loads the real checkpoint the same way)."""
    import torch
    from transformers import Qwen3VLConfig, Qwen3VLForConditionalGeneration

    s = shape
    cfg = Qwen3VLConfig(
        text_config=dict(
            hidden_size=s.hidden, num_attention_heads=s.num_heads, num_key_value_heads=s.num_kv_heads,
            head_dim=s.head_dim, intermediate_size=s.intermediate, vocab_size=s.vocab,
            num_hidden_layers=s.num_layers, rms_norm_eps=s.rms_eps,
            rope_parameters={"rope_type": "default", "rope_theta": s.rope_theta,
                             "mrope_section": list(s.mrope_section), "mrope_interleaved": True},
            max_position_embeddings=32768, attention_bias=False, hidden_act="silu",
        ),
        vision_config=dict(depth=1, hidden_size=64, intermediate_size=64, num_heads=2,
                           out_hidden_size=s.hidden, deepstack_visual_indexes=[]),
        tie_word_embeddings=True,
    )
    cfg.text_config._attn_implementation = "sdpa"
    torch.manual_seed(seed)
    model = Qwen3VLForConditionalGeneration(cfg).eval().float()
    if state is None:
        state = synthetic_state(s, seed=seed)
    lm = model.model.language_model
    lm.load_state_dict({k: v.float() for k, v in state.items()}, strict=True)
    model.lm_head.weight = lm.embed_tokens.weight  # tied (config tie_word_embeddings)
    return model
