"""Drop-in for the reference's `optimized_layer` module: an HF-compatible
decoder layer whose single-token decode step runs on the B200 kernels.

`OptimizedDecoderLayer` keeps the constructor and forward signature of the
reference's class (`optimized_layer.py:29-469`): it is built from an HF
`Qwen3VLTextDecoderLayer`, concatenates the q/k/v and gate/up weights once
(`optimized_layer.py:60-84`), and is called by HF's own layer loop with
`(hidden_states, position_embeddings, attention_mask, position_ids,
past_key_values, use_cache, cache_position, **kwargs)`.
`replace_decoder_layers(model)` swaps every text-decoder layer of a
`Qwen3VLForConditionalGeneration` in place (`optimized_layer.py:3848-3858`).

Decode step (one token, fp16 on CUDA, HF `StaticCache`): the reference's
chain of fused ops (`optimized_layer.py:156-469`), each a call of the
drop-in modules of this package:

    fused_rmsnorm_qkv_half           RMSNorm + fused QKV GEMV
    fused_q_rope_kv_cache_update     q/k RMSNorm + rotary (HF's cos/sin) + K/V written
                                     into the StaticLayer at the cache position
    decode_attn_v4_cta_qhead_splitkv_fused   split-KV GQA attention over slots [0, pos]
    nosplit_matvec_half              o_proj
    fused_post_attn_mlp_softsync_half        residual add + RMSNorm + gate/up + SiLU*up
                                     + down + residual

The cache position is `cache_position` when the caller passes it (older HF
and the reference's own eager step pass it), else the StaticLayer's
`cumulative_length` (HF 5.x), which the layer then advances by one as
`StaticLayer.update` would.  Any other input (a multi-token prefill, another
cache type, fp32, CPU) runs HF's layer math over the fused weights, as the
reference falls back to HF's modules when its fused ops decline
(`optimized_layer.py:166-179, 2344-2352`); the decode kernels themselves have
no CPU or eager fallback and raise if the native library is missing.
"""
from __future__ import annotations

import torch
import torch.nn as nn

import cuda_decode_attention
import cuda_decode_gemv
import cuda_decode_small_ops

__all__ = ["OptimizedDecoderLayer", "replace_decoder_layers"]


class OptimizedDecoderLayer(nn.Module):
    """Drop-in replacement for `Qwen3VLTextDecoderLayer` (same forward
    signature, uses the original layer's weights)."""

    def __init__(self, orig_layer):
        super().__init__()
        attn = orig_layer.self_attn
        mlp = orig_layer.mlp
        cfg = attn.config
        self.hidden_size = orig_layer.hidden_size
        self.head_dim = attn.head_dim
        self.num_heads = cfg.num_attention_heads
        self.num_kv_heads = cfg.num_key_value_heads
        self.num_key_value_groups = attn.num_key_value_groups
        self.scaling = attn.scaling
        self.layer_idx = attn.layer_idx
        self.rms_norm_eps = cfg.rms_norm_eps
        self.q_size = self.num_heads * self.head_dim
        self.kv_size = self.num_kv_heads * self.head_dim
        self.intermediate_size = mlp.intermediate_size

        self.config = cfg
        self.is_causal = True
        self.attention_dropout = attn.attention_dropout
        # HF's norm modules and activation are kept (they hold only the
        # weights the decode kernels also read), and the RMSNorm weights are
        # exposed under the reference's names
        self.input_layernorm = orig_layer.input_layernorm
        self.post_attention_layernorm = orig_layer.post_attention_layernorm
        self.q_norm = attn.q_norm
        self.k_norm = attn.k_norm
        self.act_fn = mlp.act_fn
        self.input_layernorm_weight = self.input_layernorm.weight
        self.post_attn_layernorm_weight = self.post_attention_layernorm.weight
        self.q_norm_weight = self.q_norm.weight
        self.k_norm_weight = self.k_norm.weight
        # fused projections: [q; k; v] rows and [gate; up] rows, built once
        self.qkv_weight = nn.Parameter(torch.cat([attn.q_proj.weight.data, attn.k_proj.weight.data,
                                                  attn.v_proj.weight.data], dim=0), requires_grad=False)
        self.qkv_bias = None
        if attn.q_proj.bias is not None:
            self.qkv_bias = nn.Parameter(torch.cat([attn.q_proj.bias.data, attn.k_proj.bias.data,
                                                    attn.v_proj.bias.data]), requires_grad=False)
        self.gate_up_weight = nn.Parameter(torch.cat([mlp.gate_proj.weight.data, mlp.up_proj.weight.data], dim=0),
                                           requires_grad=False)
        self.o_proj = attn.o_proj
        self.down_proj = mlp.down_proj
        self.decode_steps = 0  # forward calls served by the decode kernels (host-side count)

    @property
    def o_proj_weight(self):
        return self.o_proj.weight

    @property
    def o_proj_bias(self):
        return self.o_proj.bias

    @property
    def down_proj_weight(self):
        return self.down_proj.weight

    @property
    def down_proj_bias(self):
        return self.down_proj.bias

    # -------------------------------------------------------------- dispatch
    def _static_layer(self, past_key_values):
        """The HF StaticLayer of this layer when it is ready for the decode
        kernels (fp16 CUDA keys/values [1, KVH, Lmax, 128], contiguous), else None."""
        layers = getattr(past_key_values, "layers", None)
        if layers is None or self.layer_idx >= len(layers):
            return None
        lay = layers[self.layer_idx]
        if not getattr(lay, "is_initialized", False) or getattr(lay, "is_sliding", False):
            return None
        k, v = getattr(lay, "keys", None), getattr(lay, "values", None)
        if k is None or v is None or getattr(lay, "cumulative_length", None) is None:
            return None
        if (k.dtype != torch.float16 or v.dtype != torch.float16 or not k.is_cuda or k.dim() != 4
                or k.shape[0] != 1 or k.shape[1] != self.num_kv_heads or k.shape[-1] != self.head_dim
                or k.shape != v.shape or not k.is_contiguous() or not v.is_contiguous()):
            return None
        return lay

    def _decode_ok(self, hidden_states, position_embeddings) -> bool:
        cos, sin = position_embeddings
        return (hidden_states.is_cuda and hidden_states.dtype == torch.float16 and hidden_states.dim() == 3
                and hidden_states.shape[0] == 1 and hidden_states.shape[1] == 1
                and self.head_dim == 128 and self.num_key_value_groups == 2
                and cos.dtype == torch.float16 and sin.dtype == torch.float16
                and cos.shape[-1] == self.head_dim and cos.numel() == self.head_dim)

    def forward(self, hidden_states: torch.Tensor, position_embeddings: tuple, attention_mask=None,
                position_ids=None, past_key_values=None, use_cache=False, cache_position=None,
                **kwargs) -> torch.Tensor:
        lay = self._static_layer(past_key_values) if past_key_values is not None else None
        if lay is None or not self._decode_ok(hidden_states, position_embeddings):
            return self._hf_forward(hidden_states, position_embeddings, attention_mask, past_key_values,
                                    cache_position, **kwargs)
        return self._decode_step(hidden_states, position_embeddings, lay, cache_position)

    # -------------------------------------------------------------- other inputs
    def _hf_forward(self, hidden_states, position_embeddings, attention_mask, past_key_values, cache_position,
                    **kwargs):
        """HF's decoder-layer math (modeling_qwen3_vl.py: attention :467-505,
        MLP :519-521, layer :535-563) over the fused weights, with HF's own
        norm modules, rotary helper, cache update and attention interface:
        the path for prefill and any input the decode kernels do not take."""
        from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
        from transformers.models.qwen3_vl.modeling_qwen3_vl import apply_rotary_pos_emb, eager_attention_forward

        F = torch.nn.functional
        input_shape = hidden_states.shape[:-1]
        residual = hidden_states
        x = self.input_layernorm(hidden_states)
        qkv = F.linear(x, self.qkv_weight, self.qkv_bias)
        q, k, v = qkv.split([self.q_size, self.kv_size, self.kv_size], dim=-1)
        q = self.q_norm(q.reshape(*input_shape, -1, self.head_dim)).transpose(1, 2)
        k = self.k_norm(k.reshape(*input_shape, -1, self.head_dim)).transpose(1, 2)
        v = v.reshape(*input_shape, -1, self.head_dim).transpose(1, 2)
        cos, sin = position_embeddings
        q, k = apply_rotary_pos_emb(q, k, cos, sin)
        if past_key_values is not None:
            cache_kwargs = {"sin": sin, "cos": cos, "cache_position": cache_position}
            k, v = past_key_values.update(k, v, self.layer_idx, cache_kwargs)
        interface = ALL_ATTENTION_FUNCTIONS.get_interface(self.config._attn_implementation, eager_attention_forward)
        attn, _ = interface(self, q, k, v, attention_mask, dropout=0.0, scaling=self.scaling, **kwargs)
        h = residual + self.o_proj(attn.reshape(*input_shape, -1).contiguous())
        gate, up = F.linear(self.post_attention_layernorm(h), self.gate_up_weight).chunk(2, dim=-1)
        return h + self.down_proj(self.act_fn(gate) * up)

    # -------------------------------------------------------------- decode
    def _decode_step(self, hidden_states, position_embeddings, lay, cache_position):
        advance = cache_position is None
        pos = (lay.cumulative_length if advance else cache_position).reshape(-1)[:1]
        if pos.dtype != torch.long or pos.device != hidden_states.device:
            pos = pos.to(device=hidden_states.device, dtype=torch.long)
        eps = self.rms_norm_eps
        residual = hidden_states
        qkv = cuda_decode_gemv.fused_rmsnorm_qkv_half(hidden_states, self.input_layernorm_weight, self.qkv_weight,
                                                      self.qkv_bias, eps)
        q, k, v = qkv.split([self.q_size, self.kv_size, self.kv_size], dim=-1)
        cos, sin = position_embeddings
        q_rot = cuda_decode_small_ops.fused_q_rope_kv_cache_update(
            q.reshape(1, 1, self.num_heads, self.head_dim), k.reshape(1, 1, self.num_kv_heads, self.head_dim),
            v.reshape(1, 1, self.num_kv_heads, self.head_dim), self.q_norm_weight, self.k_norm_weight, eps,
            cos.reshape(1, 1, self.head_dim), sin.reshape(1, 1, self.head_dim), lay.keys, lay.values, pos)
        attn = cuda_decode_attention.decode_attn_v4_cta_qhead_splitkv_fused(
            q_rot.transpose(1, 2), lay.keys, lay.values, self.scaling, self.num_key_value_groups, pos)
        if attn is None:
            raise RuntimeError("decode attention declined an input the layer had accepted")
        o = cuda_decode_gemv.nosplit_matvec_half(attn.reshape(1, 1, self.q_size), self.o_proj_weight,
                                                 self.o_proj_bias)
        _act, out = cuda_decode_gemv.fused_post_attn_mlp_softsync_half(
            residual, o, self.post_attn_layernorm_weight, self.gate_up_weight, self.down_proj_weight,
            self.down_proj_bias, eps)
        if advance:
            lay.cumulative_length.add_(1)  # what StaticLayer.update does for the one new token
        self.decode_steps += 1
        return out


def replace_decoder_layers(model) -> int:
    """Replace every text-decoder layer of a Qwen3-VL model with
    OptimizedDecoderLayer (in place); returns the number replaced."""
    layers = model.model.language_model.layers
    is_eval = not model.training
    count = 0
    for i in range(len(layers)):
        if isinstance(layers[i], OptimizedDecoderLayer):
            continue
        layers[i] = OptimizedDecoderLayer(layers[i])
        if is_eval:
            layers[i].eval()
        count += 1
    return count
