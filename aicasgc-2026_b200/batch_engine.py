"""Batched greedy decode of up to 8 independent requests per step (B200).

Each decode step is ONE persistent launch of the batched phase-program
kernel (`aicas_decode_batch_f16`, csrc/decode_batch.cu) over all active
requests ("streams"): the weights stream from HBM once per step for every
stream, and each projection is an [streams, k] x [k, n] contraction on the
tensor cores (tcgen05.mma, fp16 operands, fp32 accumulation).  Streams are
ragged: each has its own prompt length, cache position, 3-axis rope position,
step state, EOS and KV cache slice, and a stream that ended is skipped.

Prompts are prefilled one request at a time with the one-pass prefill
(prefill.py, library GEMMs) straight into the stream's slice of the cache.

This is the batch-8 request-parallel configuration of the reference's decode
path: the reference's engine serves one request (`GreedyDecodeEngine`
rejects batch > 1, evaluation_wrapper.py:110-111) and its attention kernel
reads only `cache_position[0]` (cuda_extensions/decode_attention_v4_kernel.cu:
647-900); per stream, every step computes what the batch-1 step computes.

KV layout: `k_cache` / `v_cache` [layers, max_batch, num_kv_heads,
max_cache_len, 128] fp16 storage (the shape of HF `StaticLayer`s of batch
max_batch, transformers/cache_utils.py:247-354), each (layer, stream, head)
slice in the KV tile layout: slot p, dim d at element (p // 8) * 1024 +
(d // 8) * 64 + (p % 8) * 8 + d % 8, so a 64-slot chunk lands in shared
memory as a tensor-core operand with one bulk copy.  `kv_tiles` views the
storage as [.., slot groups, dim blocks, 8 slots, 8 dims], `kv_hf_layout`
returns a copy in HF's [.., slots, dims] order.
"""
from __future__ import annotations

import ctypes

import torch

from _native import (F_CNT_IN, F_CNT_OUT, F_CNT_RESID, F_KBLOCKED, F_LL_IN, F_LL_OUT, F_NORM, F_RESID,
                     F_RESID_EMBED, F_X_EMBED, MAX_BATCH, PH_ATTN, PH_GATEUP, PH_GEMV, PH_LMHEAD, AicasError,
                     AicasPhase, AicasStepState, batch_scratch_bytes, check, lib)
from _ops import device_error
from engine import hf_inv_freq
from prefill import layer_weights_from_hf, prefill
from qwen3vl_config import QWEN3VL_2B, Qwen3VLTextShape

_DONE = AicasStepState.done_step.offset // 8


def kv_tiles(cache: torch.Tensor) -> torch.Tensor:
    """View of a [L, B, KVH, Lmax, D] KV tile layout cache as [L, B, KVH,
    Lmax / 8, D / 8, 8 slots, 8 dims]."""
    L, B, H, M, D = cache.shape
    return cache.view(L, B, H, M // 8, D // 8, 8, 8)


def kv_hf_layout(cache: torch.Tensor) -> torch.Tensor:
    """A copy of a KV tile layout cache in HF's [L, B, KVH, Lmax, D] order."""
    return kv_tiles(cache).permute(0, 1, 2, 3, 5, 4, 6).reshape(cache.shape)


def kv_store_tiles(cache: torch.Tensor, b: int, src: torch.Tensor):
    """Write `src` [L, KVH, P8, D] (HF order, P8 a multiple of 8) into slots
    [0, P8) of stream b of a KV tile layout cache."""
    L, H, P8, D = src.shape
    kv_tiles(cache)[:, b, :, :P8 // 8] = src.view(L, H, P8 // 8, 8, D // 8, 8).permute(0, 1, 2, 4, 3, 5)


def tile_weight(w: torch.Tensor) -> torch.Tensor:
    """Row-major [n, k] -> the tensor-core tile layout of the batched kernel:
    [k / 2048][n / 8][256][8][8], i.e. every 8-row x 2048-column block (K
    chunk c, row group g) is 32 contiguous KB holding column group v (8
    columns) of its 8 rows at [v][row][column]; blocks are ordered chunk-major
    (the K-blocked order).  `aicas_tile_weight_f16` does the same on the
    device."""
    n, k = w.shape
    if n % 8 or k % 2048:
        raise AicasError(f"tile layout needs n % 8 == 0 and k % 2048 == 0, got {tuple(w.shape)}")
    return w.reshape(n // 8, 8, k // 2048, 256, 8).permute(2, 0, 3, 1, 4).contiguous()


class Qwen3VLBatchDecodeEngine:
    """Greedy decode of up to `max_batch` requests at once (fp16 weights,
    fp32 accumulation).  `state` maps HF text-model keys to tensors, as for
    `engine.Qwen3VLDecodeEngine`."""

    def __init__(self, state: dict, shape: Qwen3VLTextShape = QWEN3VL_2B, *, max_batch: int = MAX_BATCH,
                 max_cache_len: int = 4608, device: torch.device | str = "cuda", max_steps: int = 8192,
                 logits_ring: int = 0):
        if not 1 <= max_batch <= MAX_BATCH:
            raise AicasError(f"max_batch must be 1..{MAX_BATCH}")
        self.shape = shape
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        if max_cache_len % 64:
            max_cache_len += 64 - max_cache_len % 64
        self.max_cache_len = max_cache_len
        self.max_batch = max_batch
        self.max_steps = max_steps
        self._lib = lib()
        s, dev, B = shape, self.device, max_batch
        f16 = dict(dtype=torch.float16, device=dev)
        with torch.cuda.device(dev):
            self.embed = state["embed_tokens.weight"].to(**f16).contiguous()
            self.final_norm = state["norm.weight"].to(**f16).contiguous()
            # row-major layer weights (the prefill's GEMMs) and their tensor-core tiles (the decode step)
            self.layers = layer_weights_from_hf(state, s.num_layers, dtype=torch.float16, device=dev)
            self.tiled = [{k: tile_weight(L[k]) for k in ("qkv", "o", "gate_up", "down")} for L in self.layers]
            self.lm_tiled = tile_weight(self.embed)
            kv_shape = (s.num_layers, B, s.num_kv_heads, max_cache_len, s.head_dim)
            self.k_cache = torch.zeros(kv_shape, **f16)
            self.v_cache = torch.zeros(kv_shape, **f16)
            # qkv: LL words [stream][len] (attention polls only its heads' columns); the
            # others are counted fp16 vectors in the operand layout [len / 8][8 stream slots][8]
            self.qkv = torch.zeros((B, s.qkv_rows), dtype=torch.int32, device=dev)
            self.h = torch.zeros((s.hidden // 8, MAX_BATCH, 8), **f16)
            self.h_mid = torch.zeros((s.hidden // 8, MAX_BATCH, 8), **f16)
            self.attn = torch.zeros((s.q_size // 8, MAX_BATCH, 8), **f16)
            self.act = torch.zeros((s.intermediate // 8, MAX_BATCH, 8), **f16)
            self.out_tokens = torch.full((B, max_steps), -1, dtype=torch.int64, device=dev)
            self.logits_ring = int(logits_ring)
            self.logits = torch.zeros((B, logits_ring, s.vocab), **f16) if logits_ring > 0 else None
            self.scratch = torch.zeros(batch_scratch_bytes(), dtype=torch.uint8, device=dev)
            self.state_dev = torch.zeros((B, ctypes.sizeof(AicasStepState)), dtype=torch.uint8, device=dev)
            self.scripts = [torch.zeros((1, 5), dtype=torch.int64, device=dev) for _ in range(B)]
            self.num_ctas = self._lib.aicas_num_ctas(dev.index)
            if self.num_ctas <= 0:
                raise AicasError(f"aicas_num_ctas failed ({self.num_ctas})")
            self._inv_freq = hf_inv_freq(s)
            self._build_program()
            for b in range(B):
                self._write_state(b, 0, 0, (0, 0, 0), 0, 0, done=True)
        self.prompt_len = [0] * B
        self._graphs: dict[int, torch.cuda.CUDAGraph] = {}

    # ------------------------------------------------------------------ program
    def _build_program(self):
        """28 x [QKV, ATTN, O_PROJ, GATE_UP, DOWN] + LM_HEAD, as the batch-1
        program (engine.py), with tile-layout weights and per-stream rows.
        qkv is an LL vector (each attention CTA polls only its heads'
        columns); attn, h_mid, act and h are counted vectors (every CTA reads
        all of them, once, after all CTAs have written them).  Every GEMV
        phase gives every CTA rows (checked), so one buffer per vector can be
        reused across layers."""
        s, nct = self.shape, self.num_ctas
        eps = float(s.rms_eps)
        phases = []
        extra = 0

        def ptr(t):
            return t.data_ptr()

        def gemv_like(kind, flags, n, k, w, x, out, norm_w=None, resid=None, x_src=-1):
            nonlocal extra
            groups = n // 8
            if groups < nct:
                raise AicasError(f"phase with {groups} row groups < {nct} CTAs breaks LL buffer reuse")
            p = AicasPhase()
            p.kind, p.flags, p.n, p.k = kind, flags, n, k
            p.rot = extra % nct
            extra += groups % nct
            p.w, p.x = ptr(w), ptr(x)
            p.out = ptr(out) if out is not None else None
            p.norm_w = ptr(norm_w) if norm_w is not None else None
            p.resid = ptr(resid) if resid is not None else None
            p.embed_rows = s.vocab
            p.x_src = x_src
            p.eps = eps
            phases.append(p)

        for li, (L, T) in enumerate(zip(self.layers, self.tiled)):
            first = li == 0
            base = 5 * li
            if first:
                gemv_like(PH_GEMV, F_NORM | F_X_EMBED | F_LL_OUT, s.qkv_rows, s.hidden, T["qkv"], self.embed,
                          self.qkv, norm_w=L["ln1"])
            else:
                gemv_like(PH_GEMV, F_NORM | F_CNT_IN | F_LL_OUT, s.qkv_rows, s.hidden, T["qkv"], self.h, self.qkv,
                          norm_w=L["ln1"], x_src=base - 1)
            a = AicasPhase()
            a.kind, a.flags = PH_ATTN, F_LL_IN | F_CNT_OUT
            a.kv_heads, a.q_heads, a.max_len = s.num_kv_heads, s.num_heads, self.max_cache_len
            a.k, a.n = s.qkv_rows, s.q_size  # row lengths of the stream's qkv input and attention output
            a.x, a.out, a.x_src = ptr(self.qkv), ptr(self.attn), base
            a.norm_w, a.norm_w2 = ptr(L["qn"]), ptr(L["kn"])
            a.k_cache, a.v_cache = ptr(self.k_cache[li]), ptr(self.v_cache[li])
            a.eps, a.scale = eps, float(s.head_dim ** -0.5)
            phases.append(a)
            gemv_like(PH_GEMV, F_CNT_IN | F_CNT_OUT | F_RESID | (F_RESID_EMBED if first else F_CNT_RESID), s.hidden,
                      s.q_size, T["o"], self.attn, self.h_mid, resid=self.embed if first else self.h, x_src=base + 1)
            gemv_like(PH_GATEUP, F_NORM | F_CNT_IN | F_CNT_OUT, s.intermediate, s.hidden, T["gate_up"], self.h_mid,
                      self.act, norm_w=L["ln2"], x_src=base + 2)
            gemv_like(PH_GEMV, F_CNT_IN | F_CNT_OUT | F_RESID | F_CNT_RESID | F_KBLOCKED, s.hidden, s.intermediate,
                      T["down"], self.act, self.h, resid=self.h_mid, x_src=base + 3)
        gemv_like(PH_LMHEAD, F_NORM | F_CNT_IN, s.vocab, s.hidden, self.lm_tiled, self.h, None,
                  norm_w=self.final_norm, x_src=5 * s.num_layers - 1)
        arr = (AicasPhase * len(phases))(*phases)
        check(self._lib.aicas_validate_batch_phases(arr, len(phases)), "aicas_validate_batch_phases")
        raw = torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8)
        self.program = raw.to(self.device)
        self.n_phases = len(phases)

    # ------------------------------------------------------------------ state
    def _write_state(self, b, token, cache_pos, rope, step, script_len, eos_token=-1, done=False):
        st = AicasStepState()
        st.eos_token, st.done_step = int(eos_token), (1 if done else 0)
        st.token, st.cache_pos = int(token), int(cache_pos)
        for i in range(3):
            st.rope[i] = int(rope[i])
        st.step, st.script_len = int(step), int(script_len)
        st.script = self.scripts[b].data_ptr()
        st.out_tokens = self.out_tokens[b].data_ptr()
        st.max_steps = self.max_steps
        st.logits = self.logits[b].data_ptr() if self.logits is not None else None
        st.logits_ring = max(self.logits_ring, 1)
        for i in range(64):
            st.inv_freq[i] = float(self._inv_freq[i])
        for i in range(3):
            st.mrope_section[i] = int(self.shape.mrope_section[i])
        host = torch.frombuffer(bytearray(bytes(st)), dtype=torch.uint8)
        self.state_dev[b].copy_(host, non_blocking=False)

    def add_request(self, b: int, prompt, pos3=None, eos_token_id: int | None = None) -> int:
        """Prefill `prompt` (positions `pos3` [3, P], default text positions)
        into stream b's cache slots [0, P) in one pass and make the stream
        active; returns its first generated token (logits in the stream's
        logits ring, id in out_tokens[b, P - 1]).  With `eos_token_id` the
        stream ends on the device at its first generated EOS."""
        if not 0 <= b < self.max_batch:
            raise AicasError(f"stream {b} out of range")
        tokens = torch.as_tensor(prompt, dtype=torch.int64).reshape(-1).cpu()
        P = tokens.numel()
        if P < 1 or P >= self.max_cache_len or P > self.max_steps:
            raise AicasError("prompt does not fit the cache")
        if pos3 is None:
            pos3 = torch.arange(P, dtype=torch.int64).expand(3, P)
        pos3 = torch.as_tensor(pos3, dtype=torch.int64).reshape(3, P).cpu()
        s, dev = self.shape, self.device
        with torch.cuda.device(dev):
            # the prefill writes HF-ordered slots [0, P); they go into the
            # stream's slice in the KV tile layout (whole 8-slot groups)
            P8 = (P + 7) // 8 * 8
            kt = torch.zeros((s.num_layers, 1, s.num_kv_heads, P8, s.head_dim), dtype=torch.float16, device=dev)
            vt = torch.zeros_like(kt)
            logits = prefill(tokens.to(dev), pos3.to(dev), self.embed, self.final_norm, self.layers, kt, vt,
                             num_heads=s.num_heads, num_kv_heads=s.num_kv_heads, head_dim=s.head_dim,
                             eps=float(s.rms_eps), inv_freq=self._inv_freq.to(dev), mrope_section=s.mrope_section)
            kv_store_tiles(self.k_cache, b, kt[:, 0])
            kv_store_tiles(self.v_cache, b, vt[:, 0])
            del kt, vt
            first = int(torch.argmax(logits))
            if self.logits is not None:
                self.logits[b, (P - 1) % self.logits_ring].copy_(logits.to(torch.float16))
            self.out_tokens[b].fill_(-1)
            self.out_tokens[b, P - 1] = first
            self._write_state(b, first, P, (pos3[:, -1] + 1).tolist(), P, P,
                              -1 if eos_token_id is None else int(eos_token_id))
            if eos_token_id is not None and first == int(eos_token_id):
                self.state_dev[b].view(torch.int64)[_DONE].fill_(P)
        self.prompt_len[b] = P
        return first

    def end_request(self, b: int):
        """Make stream b inactive (its slot is skipped by every later step)."""
        self.state_dev[b].view(torch.int64)[_DONE].fill_(1)

    # ------------------------------------------------------------------ launch
    def launch(self, n: int = 1):
        """n decode steps of every active stream, eagerly."""
        stream = ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        for _ in range(n):
            rc = self._lib.aicas_decode_batch_f16(ctypes.c_void_p(self.program.data_ptr()), self.n_phases,
                                                  ctypes.c_void_p(self.state_dev.data_ptr()), self.max_batch,
                                                  ctypes.c_void_p(self.scratch.data_ptr()), stream)
            check(rc, "aicas_decode_batch_f16")

    def launch_traced(self) -> torch.Tensor:
        """One batched step with per-CTA per-phase %globaltimer stamps
        (aicas_decode_batch_trace_f16); returns trace [num_ctas, n_phases, 8]
        after synchronising."""
        trace = torch.zeros((self.num_ctas, self.n_phases, 8), dtype=torch.int64, device=self.device)
        stream = ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        rc = self._lib.aicas_decode_batch_trace_f16(ctypes.c_void_p(self.program.data_ptr()), self.n_phases,
                                                    ctypes.c_void_p(self.state_dev.data_ptr()), self.max_batch,
                                                    ctypes.c_void_p(self.scratch.data_ptr()),
                                                    ctypes.c_void_p(trace.data_ptr()), stream)
        check(rc, "aicas_decode_batch_trace_f16")
        torch.cuda.synchronize(self.device)
        return trace.cpu()

    def graph(self, steps: int) -> torch.cuda.CUDAGraph:
        """A CUDA graph of `steps` consecutive batched steps (captured once;
        replays advance the device step states)."""
        g = self._graphs.get(steps)
        if g is None:
            snap = self.state_dev.clone()
            self.launch(1)  # warm-up outside capture
            torch.cuda.synchronize(self.device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self.launch(steps)
            torch.cuda.synchronize(self.device)
            self.state_dev.copy_(snap)
            self._graphs[steps] = g
        return g

    def run(self, n: int, graph_steps: int = 32):
        if graph_steps > 1 and n >= graph_steps:
            g = self.graph(graph_steps)
            for _ in range(n // graph_steps):
                g.replay()
            n %= graph_steps
        if n:
            self.launch(n)

    # ------------------------------------------------------------------ API
    def generate_batch(self, prompts, max_new_tokens: int, pos3s=None, eos_token_id: int | None = None,
                       graph_steps: int = 32) -> list[torch.Tensor]:
        """Greedy decode of len(prompts) <= max_batch requests at once: each
        prompt is prefilled into its stream, then max_new_tokens - 1 batched
        steps run.  Returns each request's new tokens (CPU int64), ending at
        its first EOS (included) when `eos_token_id` is given."""
        if len(prompts) > self.max_batch:
            raise AicasError(f"{len(prompts)} requests > max_batch {self.max_batch}")
        for b in range(self.max_batch):
            if b < len(prompts):
                P = len(torch.as_tensor(prompts[b]).reshape(-1))
                if P + max_new_tokens - 1 > self.max_steps or P + max_new_tokens > self.max_cache_len:
                    raise AicasError("request exceeds max_steps / max_cache_len")
                self.add_request(b, prompts[b], None if pos3s is None else pos3s[b], eos_token_id)
            else:
                self.end_request(b)
        self.run(max_new_tokens - 1, graph_steps)
        self.check_error()
        outs = []
        for b in range(len(prompts)):
            P = self.prompt_len[b]
            toks = self.out_tokens[b, P - 1:P - 1 + max_new_tokens].cpu()
            done = self.done_step(b)
            if done:
                toks = toks[:done - (P - 1)]
            outs.append(toks)
        return outs

    def decode_host(self, start: torch.Tensor, n: int, out: torch.Tensor | None = None,
                    graph_steps: int = 32) -> torch.Tensor:
        """Public host-buffer decode call for all max_batch streams (each
        prefilled by add_request): `start` is a (pinned) CPU int64 tensor
        [max_batch, 5] = (token, cache_slot, t, h, w) of every stream's first
        step; runs `n` batched steps and returns the tokens [max_batch, n] in
        a (pinned) CPU tensor.  The host->device copy of the inputs and the
        device->host copy of the tokens are part of the call."""
        B = self.max_batch
        if out is None:
            out = torch.empty((B, n), dtype=torch.int64, pin_memory=True)
        if getattr(self, "_start_dev", None) is None or self._start_dev.shape[0] != B:
            self._start_dev = torch.empty((B, 5), dtype=torch.int64, device=self.device)
            self._first_slot = torch.tensor(self.prompt_len, dtype=torch.int64, device=self.device)
            self._gather = torch.arange(n, dtype=torch.int64, device=self.device)
        if self._gather.numel() != n:
            self._gather = torch.arange(n, dtype=torch.int64, device=self.device)
        self._first_slot.copy_(torch.tensor(self.prompt_len, dtype=torch.int64), non_blocking=True)
        self._start_dev.copy_(start, non_blocking=True)
        st = self.state_dev.view(torch.int64)  # [stream, state words]
        st[:, 0:5].copy_(self._start_dev)
        st[:, 5].copy_(st[:, 6])  # step restarts at the script end (the prompt length)
        st[:, _DONE].fill_(0)
        self.run(n, graph_steps)
        idx = self._first_slot[:, None] + self._gather[None, :]
        out.copy_(torch.gather(self.out_tokens, 1, idx), non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return out

    def done_step(self, b: int) -> int:
        """0 while stream b runs; s + 1 once its step s produced EOS (1 for a
        slot never started or ended by end_request)."""
        return int(self.state_dev[b].view(torch.int64)[_DONE].item())

    def cache_positions(self) -> list[int]:
        return [int(self.state_dev[b].view(torch.int64)[1].item()) for b in range(self.max_batch)]

    def step_logits(self, b: int, step: int) -> torch.Tensor:
        if self.logits is None:
            raise AicasError("engine built without a logits ring")
        return self.logits[b, step % self.logits_ring]

    def check_error(self):
        code = device_error(self.scratch)
        if code:
            self.reset_device_state()
            raise AicasError(f"device error {code}: {self._lib.aicas_error_string(code).decode()}")

    def reset_device_state(self):
        for t in (self.scratch, self.h, self.h_mid, self.qkv, self.attn, self.act):
            t.zero_()

    # ------------------------------------------------------------------ roofline
    def algorithmic_bytes(self, cache_positions) -> int:
        """Bytes one batched step must move: all weights once, plus each
        active stream's K/V of slots [0, pos) read and slot pos written."""
        s = self.shape
        return s.weight_bytes_per_step() + sum(s.kv_bytes_per_position() * (p + 1) for p in cache_positions)
