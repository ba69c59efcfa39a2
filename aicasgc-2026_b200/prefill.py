"""Causal prefill of a prompt into the decode engine's KV cache.

The decode kernel consumes one token per launch; feeding a 1024-token prompt
through it costs ~1 ms per token.  This module runs the whole prompt through
the text decoder at once, the way the reference prefills with HF's forward
(`evaluation_wrapper.py:1836-1958`, `optimized_layer.py:471-619`): per layer
the projections are plain library GEMMs over all prompt tokens (fp16 inputs,
fp32 accumulation, fp16 results on CUDA; fp32 then rounded to fp16 on the
CPU), the attention is causal softmax(q k^T s) v in fp32, and the
element-wise steps keep HF's fp16 rounding points (RMSNorm
modeling_qwen3_vl.py:398-403, q/k-norm + interleaved MRoPE :352-386 and
:427-431, SiLU-gated MLP :553-563, residual adds).  K and V land in the
engine's cache layout [L, 1, kv_heads, max_len, head_dim] at slots [0, P).

Both engines call it with CUDA tensors, which run `prefill_native` (the
library's prefill kernels, csrc/prefill_kernels.cu, between fp16 GEMMs); the
torch restatement `_prefill` runs only for CPU tensors, for the CPU parity
test against the oracle's prefill (tests/test_prefill.py), never as a
fallback of the GPU path.

Weights come in the engine's fused per-layer layout: qkv [4096, 2048] (q
rows, then k, then v), o [2048, 2048], gate_up [12288, 2048] (gate rows
first), down either [2048, 6144] or K-blocked [3, 2048, 2048] (block c holds
columns c*2048 .. c*2048+2047), plus the norm weights ln1, ln2, qn, kn.
"""
from __future__ import annotations

import torch


def _r16(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.float16).to(torch.float32)


def _linear(x16: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """fp16-valued [T, K] @ w[N, K]^T -> fp16 values (held in fp32)."""
    if x16.is_cuda:
        return (x16.to(torch.float16) @ w.t()).to(torch.float32)
    return _r16(x16.to(torch.float32) @ w.to(torch.float32).t())


def _down(act: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    if w.dim() == 2:
        return _linear(act, w)
    kc = w.shape[-1]  # K-blocked: sum the chunk products in fp32, round once
    if act.is_cuda:
        a16 = act.to(torch.float16)
        acc = sum((a16[:, c * kc:(c + 1) * kc] @ w[c].t()).to(torch.float32) for c in range(w.shape[0]))
    else:
        af = act.to(torch.float32)
        acc = sum(af[:, c * kc:(c + 1) * kc] @ w[c].to(torch.float32).t() for c in range(w.shape[0]))
    return _r16(acc)


def _rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    var = (x * x).mean(dim=-1, keepdim=True)
    n = _r16(x * torch.rsqrt(var + eps))
    return _r16(w.to(torch.float32) * n)


def mrope_cos_sin(pos3: torch.Tensor, inv_freq: torch.Tensor, section) -> tuple[torch.Tensor, torch.Tensor]:
    """Interleaved-MRoPE cos/sin [T, head_dim] (fp32 math, fp16 values):
    frequency i uses axis h when i % 3 == 1 and i < 3*section[1], axis w when
    i % 3 == 2 and i < 3*section[2], else axis t."""
    freqs = inv_freq.to(torch.float32)[None, None, :] * pos3.to(torch.float32)[:, :, None]  # [3, T, 64]
    out = freqs[0].clone()
    for axis, offset in ((1, 1), (2, 2)):
        out[:, offset:section[axis] * 3:3] = freqs[axis][:, offset:section[axis] * 3:3]
    emb = torch.cat([out, out], dim=-1)
    return _r16(torch.cos(emb)), _r16(torch.sin(emb))


def _rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    half = x.shape[-1] // 2
    rot = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
    return _r16(_r16(x * cos[:, None, :]) + _r16(rot * sin[:, None, :]))


@torch.no_grad()
def prefill(tokens: torch.Tensor, pos3: torch.Tensor, embed: torch.Tensor, final_norm: torch.Tensor,
            layers: list, k_cache: torch.Tensor, v_cache: torch.Tensor, *, num_heads: int, num_kv_heads: int,
            head_dim: int, eps: float, inv_freq: torch.Tensor, mrope_section) -> torch.Tensor:
    """Prefill `tokens` [P] (positions `pos3` [3, P]) into slots [0, P) of
    k_cache/v_cache [L, 1, KVH, Lmax, D]; returns the fp16-valued fp32 logits
    of the last prompt token [vocab].  CUDA tensors take the native path
    (prefill_native: the library's prefill kernels plus fp16 GEMMs); CPU
    tensors the torch restatement below (the CPU parity test's path)."""
    # fp16 GEMMs accumulate in fp32 (no reduced-precision split-K reductions)
    flag = torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction
    torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
    try:
        fn = prefill_native if embed.is_cuda else _prefill
        return fn(tokens, pos3, embed, final_norm, layers, k_cache, v_cache, num_heads=num_heads,
                  num_kv_heads=num_kv_heads, head_dim=head_dim, eps=eps, inv_freq=inv_freq,
                  mrope_section=mrope_section)
    finally:
        torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = flag


def _row_major_down(lw: dict) -> torch.Tensor:
    """down_proj as [hidden, inter] row-major (the decode engine keeps it
    K-blocked [k/2048][n][2048] and adds the row-major copy for the prefill)."""
    w = lw.get("down_rm", lw["down"])
    if w.dim() == 3:
        raise ValueError("prefill needs the row-major down_proj ('down_rm')")
    return w


def prefill_native(tokens, pos3, embed, final_norm, layers, k_cache, v_cache, *, num_heads, num_kv_heads, head_dim,
                   eps, inv_freq, mrope_section):
    """The prompt in one pass on the GPU, per layer:
    aicas_prefill_add_rmsnorm_f16 (residual add of the previous layer's down
    output fused with this layer's input norm), the QKV GEMM,
    aicas_prefill_qk_norm_rope_kv_f16 (q/k norm + interleaved MRoPE, K/V into
    the cache and, with q, into the attention's tile workspace),
    aicas_prefill_attention_tiles_f16 (causal flash attention on the tcgen05
    tensor cores), the o_proj GEMM, add + post-attention norm, the gate_up
    GEMM, aicas_prefill_silu_mul_f16 and the down GEMM.  The GEMMs are plain
    fp16 x fp16 -> fp16 with fp32 accumulation (torch.matmul = cuBLAS), at
    the roofline the bench reports (prefill is ~96% GEMM FLOPs)."""
    import ctypes

    from _native import check, lib

    L = lib()
    dev = embed.device
    tokens = tokens.to(dev).reshape(-1)
    P = tokens.numel()
    pos3 = pos3.to(device=dev, dtype=torch.int64).reshape(3, P).contiguous()
    inv = inv_freq.to(device=dev, dtype=torch.float32).contiguous()
    hid = embed.shape[1]
    qs = num_heads * head_dim
    max_len = k_cache.shape[-2]
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    f16 = dict(dtype=torch.float16, device=dev)
    h = embed[tokens].contiguous()
    x = torch.empty((P, hid), **f16)
    attn = torch.empty((P, qs), **f16)
    # q, k, v of a layer in the attention's tile layout (rows padded to 128:
    # the padding stays zero)
    tiles = torch.zeros(int(L.aicas_prefill_attention_workspace_bytes(P, 0, num_heads, num_kv_heads)),
                        dtype=torch.uint8, device=dev)
    act = None
    delta = None
    for li, lw in enumerate(layers):
        check(L.aicas_prefill_add_rmsnorm_f16(p(h), None if delta is None else p(delta), p(lw["ln1"]), p(h), p(x),
                                              P, hid, float(eps), stream), "aicas_prefill_add_rmsnorm_f16")
        qkv = x @ lw["qkv"].t()
        kc, vc = k_cache[li], v_cache[li]  # [1, KVH, Lmax, D]: written in place
        if not (kc.is_contiguous() and vc.is_contiguous()):
            raise ValueError("prefill writes the cache in place: each layer's K/V must be contiguous")
        check(L.aicas_prefill_qk_norm_rope_kv_f16(p(qkv), p(lw["qn"]), p(lw["kn"]), p(pos3), p(inv),
                                                  int(mrope_section[1]), int(mrope_section[2]), None, p(kc), p(vc),
                                                  P, 0, max_len, num_heads, num_kv_heads, float(eps), p(tiles),
                                                  stream),
              "aicas_prefill_qk_norm_rope_kv_f16")
        check(L.aicas_prefill_attention_tiles_f16(p(tiles), p(attn), P, 0, num_heads, num_kv_heads,
                                                  float(head_dim ** -0.5), stream), "aicas_prefill_attention_tiles_f16")
        o = attn @ lw["o"].t()
        check(L.aicas_prefill_add_rmsnorm_f16(p(h), p(o), p(lw["ln2"]), p(h), p(x), P, hid, float(eps), stream),
              "aicas_prefill_add_rmsnorm_f16")
        gu = x @ lw["gate_up"].t()
        inter = gu.shape[1] // 2
        if act is None:
            act = torch.empty((P, inter), **f16)
        check(L.aicas_prefill_silu_mul_f16(p(gu), p(act), P, inter, stream), "aicas_prefill_silu_mul_f16")
        delta = act @ _row_major_down(lw).t()
    # last token: residual add + final norm + tied lm_head
    xl = torch.empty((1, hid), **f16)
    check(L.aicas_prefill_add_rmsnorm_f16(p(h[-1:]), p(delta[-1:]), p(final_norm), None, p(xl), 1, hid, float(eps),
                                          stream), "aicas_prefill_add_rmsnorm_f16")
    return (xl @ embed.t())[0].to(torch.float32)


def _prefill(tokens, pos3, embed, final_norm, layers, k_cache, v_cache, *, num_heads, num_kv_heads, head_dim, eps,
             inv_freq, mrope_section):
    dev = embed.device
    tokens = tokens.to(dev).reshape(-1)
    P = tokens.numel()
    pos3 = pos3.to(dev).reshape(3, P)
    cos, sin = mrope_cos_sin(pos3, inv_freq.to(dev), mrope_section)
    h = embed[tokens].to(torch.float32)
    qs, ks = num_heads * head_dim, num_kv_heads * head_dim
    g = num_heads // num_kv_heads
    scale = head_dim ** -0.5
    causal = torch.ones((P, P), dtype=torch.bool, device=dev).tril()
    for li, lw in enumerate(layers):
        x = _rms_norm(h, lw["ln1"], eps)
        qkv = _linear(x, lw["qkv"])
        q = qkv[:, :qs].reshape(P, num_heads, head_dim)
        k = qkv[:, qs:qs + ks].reshape(P, num_kv_heads, head_dim)
        v = qkv[:, qs + ks:qs + 2 * ks].reshape(P, num_kv_heads, head_dim)
        q = _rope(_rms_norm(q, lw["qn"], eps), cos, sin)
        k = _rope(_rms_norm(k, lw["kn"], eps), cos, sin)
        k_cache[li, 0, :, :P] = k.transpose(0, 1).to(k_cache.dtype)
        v_cache[li, 0, :, :P] = v.transpose(0, 1).to(v_cache.dtype)
        kr = k.repeat_interleave(g, dim=1).transpose(0, 1)  # [H, P, D]
        vr = v.repeat_interleave(g, dim=1).transpose(0, 1)
        s = (q.transpose(0, 1) @ kr.transpose(1, 2)) * scale  # [H, P, P] fp32
        s = s.masked_fill(~causal, float("-inf"))
        p = torch.softmax(s, dim=-1)
        attn = _r16((p @ vr).transpose(0, 1).reshape(P, qs))
        h = _r16(h + _linear(attn, lw["o"]))
        x = _rms_norm(h, lw["ln2"], eps)
        gu = _linear(x, lw["gate_up"])
        inter = gu.shape[1] // 2
        gt, up = gu[:, :inter], gu[:, inter:]
        act = _r16(_r16(gt / (1.0 + torch.exp(-gt))) * up)
        h = _r16(h + _down(act, lw["down"]))
    hn = _rms_norm(h[-1:], final_norm, eps)
    return _linear(hn, embed)[0]


def layer_weights_from_hf(state: dict, num_layers: int, dtype=torch.float16, device="cpu") -> list:
    """The engine's fused per-layer layout from an HF text-model state dict
    (down kept unblocked)."""
    out = []
    for i in range(num_layers):
        p = f"layers.{i}."

        def t(k):
            return state[p + k].to(device=device, dtype=dtype)

        out.append({
            "ln1": t("input_layernorm.weight"), "ln2": t("post_attention_layernorm.weight"),
            "qn": t("self_attn.q_norm.weight"), "kn": t("self_attn.k_norm.weight"),
            "qkv": torch.cat([t("self_attn.q_proj.weight"), t("self_attn.k_proj.weight"),
                              t("self_attn.v_proj.weight")], 0),
            "o": t("self_attn.o_proj.weight"),
            "gate_up": torch.cat([t("mlp.gate_proj.weight"), t("mlp.up_proj.weight")], 0),
            "down": t("mlp.down_proj.weight"),
        })
    return out
