"""CPU oracle for the Qwen3-VL-2B text-decoder decode step — TEST INFRASTRUCTURE.

This file is the checker, never the product: only `tests/`,
`__graft_entry__.smoke()` and `bench.py`'s CPU-baseline leg may import it.  The
engine under `aicasgc-2026_b200/` never calls it and has no CPU fallback.

It restates, in numpy, the arithmetic of the path the reference runs for one
decode token (`evaluation_wrapper.py:941-952` `DecodeCudaGraphRunner._run_step`
-> HF `Qwen3VLForConditionalGeneration.forward` -> 28 x
`OptimizedDecoderLayer.forward` (`optimized_layer.py:108-469`) -> final norm ->
tied `lm_head` (`evaluation_wrapper.py:1227-1240`) -> `torch.argmax`
(`evaluation_wrapper.py:952`)).  The per-op semantics are those of the HF
modules the reference's fused kernels replace (installed
`transformers/models/qwen3_vl/modeling_qwen3_vl.py`, transformers 5.5.0):

* RMSNorm                      `modeling_qwen3_vl.py:389-403`
* rotary inv_freq              `modeling_qwen3_vl.py:322-347`
* interleaved MRoPE cos/sin    `modeling_qwen3_vl.py:350-386`
* apply_rotary_pos_emb         `modeling_qwen3_vl.py:124-128, 410-432`
* attention (q/k norm, GQA)    `modeling_qwen3_vl.py:467-505`
* MLP (SiLU(gate) * up, down)  `modeling_qwen3_vl.py:519-521`
* decoder layer residuals      `modeling_qwen3_vl.py:535-563`

Two arithmetic modes:

* ``"fp32"``: every tensor in float32 — the reference's CPU path (HF fp32,
  `GreedyDecodeEngine` with ENABLE_CUDAGRAPH=0, `evaluation_wrapper.py:513-539`).
  Pinned against golden vectors that the reference itself produced
  (`tests/golden/make_golden.py`).
* ``"fp16"``: the fp16 model as HF runs it on a GPU — weights and every
  intermediate tensor HF materialises are rounded to fp16 at the same points
  (matmul / reduction arithmetic itself stays fp32, as cuBLAS and SDPA do).
  This is the checker for the fp16 CUDA engine.

``accumulate="f64"`` (fp16 mode only) carries out the matmuls, attention and
norm reductions in float64 before each fp16 rounding point: the fp16 model
with exact sums.  Any fp32-accumulating implementation (cuBLAS, the CUDA
engine, numpy's fp32 BLAS) flips an fp16 rounding now and then where its sum
lands next to a rounding boundary, and at 28 layers those one-ulp flips move
the logits by up to ~0.02.  Two fp32 implementations compared with each other
show both sets of flips; against the exact sums only the implementation's own
remain, which is the comparison the 28-layer GPU parity test makes.

Attention is causal over the static cache prefix `[0, cache_position]`, the
contract of the reference's kernels (`decode_attention_v4_kernel.cu` reads
`valid_len = cache_position + 1`).
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


def _r16(x: np.ndarray) -> np.ndarray:
    """Round to fp16 and back (the value an fp16 tensor would hold)."""
    return x.astype(np.float16).astype(F32)


def _rnd(x: np.ndarray, mode: str) -> np.ndarray:
    return _r16(x) if mode == "fp16" else x.astype(F32, copy=False)


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float, mode: str = "fp16", acc=F32) -> np.ndarray:
    """`Qwen3VLTextRMSNorm.forward` (modeling_qwen3_vl.py:398-403) over the
    last axis: fp32 variance and scale (`acc` float64: exact), cast back to
    the activation dtype, then the weight multiply in the activation dtype."""
    xf = x.astype(acc)
    var = np.mean(xf * xf, axis=-1, keepdims=True, dtype=acc)
    n = _rnd(xf * (acc(1.0) / np.sqrt(var + acc(eps))), mode)
    return _rnd(w * n, mode)


def rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, mode: str = "fp16") -> np.ndarray:
    """x*cos + rotate_half(x)*sin with a rounding per op in fp16 mode
    (modeling_qwen3_vl.py:124-128, 427-431).  x [T, H, D], cos/sin [T, D]."""
    half = x.shape[-1] // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    c = cos[:, None, :]
    s = sin[:, None, :]
    return _rnd(_rnd(x * c, mode) + _rnd(rot * s, mode), mode)


class Qwen3VLOracle:
    """Numpy restatement of the Qwen3-VL text decoder (decode + causal prefill).

    `state` maps HF text-model keys (``embed_tokens.weight``,
    ``layers.{i}.self_attn.q_proj.weight``, ...) to arrays or torch tensors.
    """

    def __init__(self, state: dict, num_layers: int, *, mode: str = "fp32",
                 max_cache_len: int = 2048, num_heads: int = 16, num_kv_heads: int = 8,
                 head_dim: int = 128, eps: float = 1e-6, rope_theta: float = 5e6,
                 mrope_section=(24, 20, 20), inv_freq=None, accumulate: str = "f32"):
        if mode not in ("fp32", "fp16"):
            raise ValueError(mode)
        if accumulate not in ("f32", "f64") or (accumulate == "f64" and mode != "fp16"):
            raise ValueError(f"accumulate={accumulate!r} (float64 sums are an fp16-mode option)")
        self.mode = mode
        self.acc = np.float64 if accumulate == "f64" else F32
        self.L = num_layers
        self.nh, self.nkv, self.d = num_heads, num_kv_heads, head_dim
        self.eps = F32(eps)
        self.mrope_section = tuple(mrope_section)
        self.max_cache_len = max_cache_len

        def arr(key):
            t = state[key]
            if hasattr(t, "detach"):
                t = t.detach().float().cpu().numpy()
            a = np.ascontiguousarray(np.asarray(t, dtype=F32))
            a = _r16(a) if mode == "fp16" else a
            return a.astype(self.acc) if self.acc is not F32 else a

        self.embed = arr("embed_tokens.weight")
        self.final_norm = arr("norm.weight")
        self.layers = []
        for i in range(num_layers):
            p = f"layers.{i}."
            self.layers.append({
                "ln1": arr(p + "input_layernorm.weight"),
                "wq": arr(p + "self_attn.q_proj.weight"),
                "wk": arr(p + "self_attn.k_proj.weight"),
                "wv": arr(p + "self_attn.v_proj.weight"),
                "wo": arr(p + "self_attn.o_proj.weight"),
                "qn": arr(p + "self_attn.q_norm.weight"),
                "kn": arr(p + "self_attn.k_norm.weight"),
                "ln2": arr(p + "post_attention_layernorm.weight"),
                "wg": arr(p + "mlp.gate_proj.weight"),
                "wu": arr(p + "mlp.up_proj.weight"),
                "wd": arr(p + "mlp.down_proj.weight"),
            })
        # inv_freq = 1 / theta^(2i/d) in fp32 (modeling_qwen3_vl.py:343-346)
        expo = np.arange(0, head_dim, 2, dtype=np.int64).astype(F32) / F32(head_dim)
        self.inv_freq = (F32(1.0) / np.power(F32(rope_theta), expo)).astype(F32)
        if inv_freq is not None:  # e.g. the table HF computes with torch (1-ulp pow differences)
            self.inv_freq = np.asarray(inv_freq, dtype=F32).reshape(-1)
        self.k_cache = np.zeros((num_layers, num_kv_heads, max_cache_len, head_dim), self.acc)
        self.v_cache = np.zeros_like(self.k_cache)

    # ---- elementwise helpers -------------------------------------------------
    def _round(self, x):
        return _rnd(x, self.mode)

    def rms_norm(self, x: np.ndarray, w: np.ndarray) -> np.ndarray:
        return rms_norm(x, w, self.eps, self.mode, self.acc)

    def mrope_cos_sin(self, pos3: np.ndarray):
        """Interleaved-MRoPE cos/sin for positions `pos3` [3, T] (t, h, w).

        `Qwen3VLTextRotaryEmbedding.forward` + `apply_interleaved_mrope`
        (modeling_qwen3_vl.py:352-386): frequency slot i takes its position
        from axis H when i % 3 == 1 and i < 3*section[1], from W when
        i % 3 == 2 and i < 3*section[2], else from T; the 64 frequencies are
        duplicated to 128 lanes; cos/sin are fp32 then cast to the model dtype.
        """
        pos3 = np.asarray(pos3, dtype=np.int64).reshape(3, -1)
        freqs = self.inv_freq[None, None, :] * pos3.astype(F32)[:, :, None]  # [3, T, 64]
        out = freqs[0].copy()
        for axis, offset in ((1, 1), (2, 2)):
            idx = slice(offset, self.mrope_section[axis] * 3, 3)
            out[:, idx] = freqs[axis][:, idx]
        emb = np.concatenate([out, out], axis=-1).astype(F32)
        return self._round(np.cos(emb)), self._round(np.sin(emb))

    def _rope(self, x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
        return rope(x, cos, sin, self.mode)

    def _linear(self, x: np.ndarray, w: np.ndarray) -> np.ndarray:
        return self._round(x.astype(w.dtype, copy=False) @ w.T)

    # ---- model ---------------------------------------------------------------
    def forward(self, tokens, pos3, cache_start: int, *, all_logits: bool = False):
        """Run T tokens at cache slots [cache_start, cache_start+T) with causal
        attention over the cache prefix; returns the last row of logits
        (or all rows with `all_logits`).  T == 1 is one decode step."""
        tokens = np.asarray(tokens, dtype=np.int64).reshape(-1)
        T = tokens.shape[0]
        end = cache_start + T
        if end > self.max_cache_len:
            raise ValueError("cache overflow")
        cos, sin = self.mrope_cos_sin(pos3)
        h = self.embed[tokens].astype(F32)
        acc = self.acc
        scale = acc(self.d ** -0.5)
        g = self.nh // self.nkv
        for li, lw in enumerate(self.layers):
            x = self.rms_norm(h, lw["ln1"])
            q = self._linear(x, lw["wq"]).reshape(T, self.nh, self.d)
            k = self._linear(x, lw["wk"]).reshape(T, self.nkv, self.d)
            v = self._linear(x, lw["wv"]).reshape(T, self.nkv, self.d)
            q = self._rope(self.rms_norm(q, lw["qn"]), cos, sin)
            k = self._rope(self.rms_norm(k, lw["kn"]), cos, sin)
            self.k_cache[li, :, cache_start:end] = k.transpose(1, 0, 2)
            self.v_cache[li, :, cache_start:end] = v.transpose(1, 0, 2)
            K = self.k_cache[li, :, :end]  # [nkv, end, D]
            V = self.v_cache[li, :, :end]
            attn = np.empty((T, self.nh, self.d), F32)
            # query t sees keys [0, cache_start + t]
            causal = np.arange(end)[None, :] <= (cache_start + np.arange(T))[:, None]
            for hq in range(self.nh):
                kv = hq // g
                s = (q[:, hq, :].astype(acc) @ K[kv].T) * scale  # [T, end]
                s = np.where(causal, s, -np.inf).astype(acc)
                m = s.max(axis=-1, keepdims=True)
                p = np.exp(s - m).astype(acc)
                attn[:, hq, :] = (p @ V[kv]) / p.sum(axis=-1, keepdims=True, dtype=acc)
            attn = self._round(attn).reshape(T, self.nh * self.d)
            h = self._round(h + self._linear(attn, lw["wo"]))
            x = self.rms_norm(h, lw["ln2"])
            gt = self._linear(x, lw["wg"])
            up = self._linear(x, lw["wu"])
            gt_a = gt.astype(acc)
            act = self._round(self._round(gt_a / (acc(1.0) + np.exp(-gt_a))) * up)
            h = self._round(h + self._linear(act, lw["wd"]))
        hn = self.rms_norm(h if all_logits else h[-1:], self.final_norm)
        logits = self._linear(hn, self.embed)
        return logits if all_logits else logits[-1]

    def prefill(self, tokens, pos3, chunk: int = 256):
        """Causal prefill of a prompt from slot 0 (chunked to bound memory);
        returns the logits of the last prompt token."""
        tokens = np.asarray(tokens, dtype=np.int64).reshape(-1)
        pos3 = np.asarray(pos3, dtype=np.int64).reshape(3, -1)
        logits = None
        for s in range(0, tokens.shape[0], chunk):
            e = min(tokens.shape[0], s + chunk)
            logits = self.forward(tokens[s:e], pos3[:, s:e], s)
        return logits

    def decode_step(self, token: int, cache_position: int, pos3) -> np.ndarray:
        return self.forward([token], np.asarray(pos3, dtype=np.int64).reshape(3, 1), cache_position)

    def greedy(self, prompt, n_new: int, pos3_prompt=None, rope_delta: int = 0,
               forced=None):
        """Greedy decode like `GreedyDecodeEngine.generate`
        (`evaluation_wrapper.py:149-315`): prefill, argmax, then `n_new - 1`
        decode steps at cache slot `pos` with rope positions `pos + rope_delta`
        on all three axes (`evaluation_wrapper.py:507-511`).

        `forced` (optional token list) teacher-forces the input of each decode
        step, so the logits of another implementation's trajectory can be
        checked step by step.  Returns (tokens [n_new], logits [n_new, V])."""
        prompt = np.asarray(prompt, dtype=np.int64).reshape(-1)
        P = prompt.shape[0]
        if pos3_prompt is None:
            pos3_prompt = np.broadcast_to(np.arange(P, dtype=np.int64), (3, P))
        logits = self.prefill(prompt, pos3_prompt)
        toks, all_logits = [], []
        for step in range(n_new):
            tok = int(np.argmax(logits))
            toks.append(tok)
            all_logits.append(logits)
            if step == n_new - 1:
                break
            inp = tok if forced is None else int(forced[step])
            pos = P + step
            logits = self.decode_step(inp, pos, np.full((3, 1), pos + rope_delta, np.int64))
        return np.asarray(toks, dtype=np.int64), np.stack(all_logits)


def attention_reference(q: np.ndarray, k: np.ndarray, v: np.ndarray, valid_len: int,
                        scaling: float) -> np.ndarray:
    """GQA decode attention over the first `valid_len` cache slots.

    Restates `_hf_repeat_kv_attention` (`bench_decode_attention.py:241-261`):
    K/V heads are repeated to the query heads, then softmax(q K^T * s) V in
    fp32.  q [H, D], k/v [KVH, Lmax, D] -> out [H, D]."""
    H = q.shape[0]
    g = H // k.shape[0]
    out = np.empty((H, q.shape[1]), F32)
    for h in range(H):
        K = k[h // g, :valid_len].astype(F32)
        V = v[h // g, :valid_len].astype(F32)
        s = (K @ q[h].astype(F32)) * F32(scaling)
        p = np.exp(s - s.max()).astype(F32)
        out[h] = (p @ V) / p.sum(dtype=F32)
    return out


def post_attn_mlp_reference(resid, attn, norm_w, w_gate_up, w_down, eps=1e-6):
    """Reference semantics of `fused_post_attn_mlp_softsync_half`
    (cuda_decode_gemv_ops/fused.py:261-337) with HF's fp16 rounding points
    (modeling_qwen3_vl.py:519-521, 553-563): h = resid + attn;
    act = silu(gate(norm h)) * up(norm h); out = h + down(act)."""
    h = _r16(resid.astype(F32) + attn.astype(F32))
    x = rms_norm(h, norm_w, eps)
    inter = w_down.shape[1]
    g = _r16(w_gate_up[:inter].astype(F32) @ x)
    u = _r16(w_gate_up[inter:].astype(F32) @ x)
    act = _r16(_r16(g / (F32(1.0) + np.exp(-g))) * u)
    out = _r16(h + _r16(w_down.astype(F32) @ act))
    return act, out


def gemv_reference(w: np.ndarray, x: np.ndarray, round_fp16: bool = True) -> np.ndarray:
    """fp32-accumulated y = W x (what `F.linear` computes for an fp16 decode
    GEMV, `bench_decode_linears.py` compares the reference kernels with it)."""
    y = w.astype(F32) @ x.astype(F32)
    return _r16(y) if round_fp16 else y
