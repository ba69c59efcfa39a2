"""B200 decode engine for the Qwen3-VL-2B text decoder.

One decode step = ONE persistent launch of the phase-program kernel
(`aicas_decode_program_f16`): 28 x [RMSNorm+QKV, q/k-norm+MRoPE+KV-write+
split-KV attention, o_proj+residual, RMSNorm+gate_up+SiLU*up,
down+residual] + final RMSNorm + tied lm_head + argmax: 141 phases with no
grid barrier between them.  Each phase polls the flag-in-data words of the
vector it consumes (every 32-bit word carries an fp16 value and the epoch of
the phase that wrote it), so a CTA starts a phase as soon as its own inputs
are complete; weights are streamed by bulk async copies ahead of the
consumers, independently of the activations.

The step reads its inputs (token, cache slot, 3-axis rope position) from a
device-resident step state and advances it itself, so a run of N steps is N
back-to-back launches with no host work between them, captured once in a
CUDA graph.  A prompt is fed as a "script" of forced inputs: one step per
prompt token, whose argmax outputs are ignored until the script ends.

This replaces, in the reference: `GreedyDecodeEngine.generate`'s hot loop
(evaluation_wrapper.py:278-313), `DecodeCudaGraphRunner` replay/_run_step
(evaluation_wrapper.py:788-791, 941-960), HF's layer loop with
`OptimizedDecoderLayer.forward` (optimized_layer.py:108-469), the patched
lm_head (evaluation_wrapper.py:1210-1245) and `torch.argmax` (:952).

KV layout: per layer `keys/values [1, num_kv_heads, max_cache_len, 128]` fp16,
the layout of HF `StaticLayer` (transformers/cache_utils.py:247-354) that the
reference's kernels index.
"""
from __future__ import annotations

import ctypes
import math

import torch

from _native import (F_KBLOCKED, F_LL_IN, F_LL_OUT, F_LL_RESID, F_NORM, F_RESID, F_RESID_EMBED, F_X_EMBED,
                     PH_ATTN, PH_GATEUP, PH_GEMV, PH_LMHEAD, PROGRAM_LEAN, AicasError, AicasPhase, AicasStepState,
                     check, lib, scratch_bytes)
from _ops import device_error
from qwen3vl_config import QWEN3VL_2B, Qwen3VLTextShape


def hf_inv_freq(shape: Qwen3VLTextShape) -> torch.Tensor:
    """Rotary inverse frequencies computed exactly as HF does (CPU fp32,
    modeling_qwen3_vl.py:343-346)."""
    d = shape.head_dim
    return 1.0 / (shape.rope_theta ** (torch.arange(0, d, 2, dtype=torch.int64).to(dtype=torch.float) / d))


class Qwen3VLDecodeEngine:
    """Batch-1 greedy decode engine (fp16 weights, fp32 accumulation).

    `state` maps HF text-model keys (see `qwen3vl_config.synthetic_state`) to
    tensors on any device / dtype; they are converted to fp16 on `device`.
    """

    def __init__(self, state: dict, shape: Qwen3VLTextShape = QWEN3VL_2B, *, max_cache_len: int = 2048,
                 device: torch.device | str = "cuda", max_steps: int = 8192, logits_ring: int = 0):
        self.shape = shape
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        if max_cache_len % 32:
            max_cache_len += 32 - max_cache_len % 32
        self.max_cache_len = max_cache_len
        self.max_steps = max_steps
        self._lib = lib()
        dev = self.device
        f16 = dict(dtype=torch.float16, device=dev)
        s = shape

        def W(key):
            return state[key].to(**f16).contiguous()

        def kblock(w):
            n, k = w.shape
            return w.view(n, k // 2048, 2048).permute(1, 0, 2).contiguous()

        with torch.cuda.device(dev):
            self.embed = W("embed_tokens.weight")
            self.final_norm = W("norm.weight")
            self.layers = []
            for i in range(s.num_layers):
                p = f"layers.{i}."
                self.layers.append({
                    "ln1": W(p + "input_layernorm.weight"),
                    "qkv": torch.cat([W(p + "self_attn.q_proj.weight"), W(p + "self_attn.k_proj.weight"),
                                      W(p + "self_attn.v_proj.weight")], 0).contiguous(),
                    "qn": W(p + "self_attn.q_norm.weight"),
                    "kn": W(p + "self_attn.k_norm.weight"),
                    "o": W(p + "self_attn.o_proj.weight"),
                    "ln2": W(p + "post_attention_layernorm.weight"),
                    "gate_up": torch.cat([W(p + "mlp.gate_proj.weight"), W(p + "mlp.up_proj.weight")],
                                         0).contiguous(),
                    # K-blocked [k/2048][n][2048]: every 8-row tile is one contiguous 32 KB copy
                    "down": kblock(W(p + "mlp.down_proj.weight")),
                    # row-major copy for the prompt prefill's GEMM
                    "down_rm": W(p + "mlp.down_proj.weight"),
                })
            # StaticCache-layout KV: [layers][1, KVH, Lmax, 128]
            kv_shape = (s.num_layers, 1, s.num_kv_heads, max_cache_len, s.head_dim)
            self.k_cache = torch.zeros(kv_shape, **f16)
            self.v_cache = torch.zeros(kv_shape, **f16)
            # activations between phases as LL vectors: word i = {fp16 value i, uint16 epoch}
            ll = dict(dtype=torch.int32, device=dev)
            self.h = torch.zeros(s.hidden, **ll)
            self.h_mid = torch.zeros(s.hidden, **ll)
            self.qkv = torch.zeros(s.qkv_rows, **ll)
            self.attn = torch.zeros(s.q_size, **ll)
            self.act = torch.zeros(s.intermediate, **ll)
            self.out_tokens = torch.full((max_steps,), -1, dtype=torch.int64, device=dev)
            self.logits_ring = int(logits_ring)
            self.logits = (torch.zeros((logits_ring, s.vocab), **f16) if logits_ring > 0 else None)
            self.scratch = torch.zeros(scratch_bytes(), dtype=torch.uint8, device=dev)
            self.state_dev = torch.zeros(ctypes.sizeof(AicasStepState), dtype=torch.uint8, device=dev)
            self.script = torch.zeros((1, 5), dtype=torch.int64, device=dev)
            self.num_ctas = self._lib.aicas_num_ctas(dev.index)
            if self.num_ctas <= 0:
                raise AicasError(f"aicas_num_ctas failed ({self.num_ctas})")
            self._build_program()
        self._graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self._start_dev = None
        self.script_len = 0
        self._inv_freq = hf_inv_freq(s)

    # ------------------------------------------------------------------ program
    def _build_program(self):
        """28 x [QKV, ATTN, O_PROJ, GATE_UP, DOWN] + LM_HEAD.  Activations flow
        through LL vectors (each phase polls exactly the words it consumes),
        so the program has no grid barrier at all.  Reusing one buffer per
        vector is safe because every GEMV phase gives every CTA rows to
        compute (checked below) and each GEMV consumes a whole vector: no CTA
        can write a buffer again before every CTA has consumed it."""
        s, nct = self.shape, self.num_ctas
        eps = float(s.rms_eps)
        phases = []
        extra = 0

        def ptr(t):
            return t.data_ptr()

        def gemv_like(kind, flags, n, k, w, x, out, norm_w=None, resid=None, x_src=-1):
            nonlocal extra
            groups = -(-n // 8)
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

        for li, L in enumerate(self.layers):
            first = li == 0
            base = 5 * li
            if first:
                gemv_like(PH_GEMV, F_NORM | F_X_EMBED | F_LL_OUT, s.qkv_rows, s.hidden, L["qkv"], self.embed,
                          self.qkv, norm_w=L["ln1"])
            else:
                gemv_like(PH_GEMV, F_NORM | F_LL_IN | F_LL_OUT, s.qkv_rows, s.hidden, L["qkv"], self.h, self.qkv,
                          norm_w=L["ln1"], x_src=base - 1)
            a = AicasPhase()
            a.kind, a.flags = PH_ATTN, F_LL_IN | F_LL_OUT
            a.kv_heads, a.q_heads, a.max_len = s.num_kv_heads, s.num_heads, self.max_cache_len
            a.x, a.out, a.x_src = ptr(self.qkv), ptr(self.attn), base
            a.norm_w, a.norm_w2 = ptr(L["qn"]), ptr(L["kn"])
            a.k_cache, a.v_cache = ptr(self.k_cache[li]), ptr(self.v_cache[li])
            a.eps, a.scale = eps, float(s.head_dim ** -0.5)
            phases.append(a)
            gemv_like(PH_GEMV, F_LL_IN | F_LL_OUT | F_RESID | (F_RESID_EMBED if first else F_LL_RESID), s.hidden,
                      s.q_size, L["o"], self.attn, self.h_mid, resid=self.embed if first else self.h, x_src=base + 1)
            gemv_like(PH_GATEUP, F_NORM | F_LL_IN | F_LL_OUT, s.intermediate, s.hidden, L["gate_up"], self.h_mid,
                      self.act, norm_w=L["ln2"], x_src=base + 2)
            gemv_like(PH_GEMV, F_LL_IN | F_LL_OUT | F_RESID | F_LL_RESID | F_KBLOCKED, s.hidden, s.intermediate,
                      L["down"], self.act, self.h, resid=self.h_mid, x_src=base + 3)
        gemv_like(PH_LMHEAD, F_NORM | F_LL_IN, s.vocab, s.hidden, self.embed, self.h, None, norm_w=self.final_norm,
                  x_src=5 * s.num_layers - 1)
        arr = (AicasPhase * len(phases))(*phases)
        check(self._lib.aicas_validate_phases(arr, len(phases)), "aicas_validate_phases")
        # the lean kernel (no code for tile paths this program never takes)
        # when every GEMV phase qualifies: the 28-layer Qwen3-VL program does
        self.program_flags = PROGRAM_LEAN if self._lib.aicas_lean_program_ok(arr, len(phases), self.num_ctas) == 0 else 0
        raw = torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8)
        self.program = raw.to(self.device)
        self.n_phases = len(phases)

    # ------------------------------------------------------------------ state
    def _write_state(self, token, cache_pos, rope, step, script_len, eos_token=-1):
        st = AicasStepState()
        st.eos_token, st.done_step = int(eos_token), 0
        st.token, st.cache_pos = int(token), int(cache_pos)
        for i in range(3):
            st.rope[i] = int(rope[i])
        st.step, st.script_len = int(step), int(script_len)
        st.script = self.script.data_ptr()
        st.out_tokens = self.out_tokens.data_ptr()
        st.max_steps = self.max_steps
        st.logits = self.logits.data_ptr() if self.logits is not None else None
        st.logits_ring = max(self.logits_ring, 1)
        for i in range(64):
            st.inv_freq[i] = float(self._inv_freq[i])
        for i in range(3):
            st.mrope_section[i] = int(self.shape.mrope_section[i])
        host = torch.frombuffer(bytearray(bytes(st)), dtype=torch.uint8)
        self.state_dev.copy_(host, non_blocking=False)

    def load_script(self, tokens, pos3=None, start_slot: int = 0, eos_token_id: int | None = None):
        """Forced inputs for the next len(tokens) steps: token i goes to cache
        slot start_slot + i with rope positions pos3[:, i] (default: the slot
        on all three axes).  After the script the engine decodes greedily
        from slot start_slot + len(tokens), rope positions advancing by one.
        With `eos_token_id`, the device ends the request at the first
        generated token equal to it: every later launch returns at once."""
        tokens = torch.as_tensor(tokens, dtype=torch.int64).reshape(-1).cpu()
        P = tokens.numel()
        if P < 1 or start_slot + P > self.max_cache_len:
            raise AicasError("script does not fit the cache")
        slots = torch.arange(start_slot, start_slot + P, dtype=torch.int64)
        if pos3 is None:
            pos3 = slots.expand(3, P)
        pos3 = torch.as_tensor(pos3, dtype=torch.int64).reshape(3, P).cpu()
        script = torch.stack([tokens, slots, pos3[0], pos3[1], pos3[2]], 1).contiguous()
        self.script = script.to(self.device)
        self.out_tokens.fill_(-1)
        self._write_state(script[0, 0], script[0, 1], script[0, 2:5], 0, P,
                          -1 if eos_token_id is None else int(eos_token_id))
        self.script_len = P

    # ------------------------------------------------------------------ launch
    def launch(self, n: int = 1):
        """n decode steps, eagerly (no graph)."""
        stream = ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        for _ in range(n):
            rc = self._lib.aicas_decode_program_ex_f16(ctypes.c_void_p(self.program.data_ptr()), self.n_phases,
                                                       ctypes.c_void_p(self.state_dev.data_ptr()),
                                                       ctypes.c_void_p(self.scratch.data_ptr()), None,
                                                       self.program_flags, stream)
            check(rc, "aicas_decode_program_ex_f16")

    def launch_traced(self) -> torch.Tensor:
        """One step with per-CTA per-phase %globaltimer stamps; returns the
        trace [num_ctas, n_phases, 8] (start, inputs ready, end, consumer
        tile-wait ns, producer slot-wait ns, tiles, compute done, results
        issued) after synchronising."""
        trace = torch.zeros((self.num_ctas, self.n_phases, 8), dtype=torch.int64, device=self.device)
        stream = ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        rc = self._lib.aicas_decode_program_ex_f16(ctypes.c_void_p(self.program.data_ptr()), self.n_phases,
                                                   ctypes.c_void_p(self.state_dev.data_ptr()),
                                                   ctypes.c_void_p(self.scratch.data_ptr()),
                                                   ctypes.c_void_p(trace.data_ptr()), self.program_flags, stream)
        check(rc, "aicas_decode_program_ex_f16")
        torch.cuda.synchronize(self.device)
        return trace.cpu()

    def phase_names(self) -> list[str]:
        names = []
        for li in range(self.shape.num_layers):
            names += [f"L{li}.qkv", f"L{li}.attn", f"L{li}.o_proj", f"L{li}.gate_up", f"L{li}.down"]
        return names + ["lm_head"]

    def graph(self, steps: int) -> torch.cuda.CUDAGraph:
        """A CUDA graph of `steps` consecutive decode steps (captured once;
        replays advance the device step state)."""
        g = self._graphs.get(steps)
        if g is None:
            snap = self.snapshot()
            self.launch(1)  # warm-up outside capture
            torch.cuda.synchronize(self.device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self.launch(steps)
            torch.cuda.synchronize(self.device)
            self.restore(snap)
            self._graphs[steps] = g
        return g

    def run(self, n: int, graph_steps: int = 32):
        """n steps using graphs of `graph_steps` launches plus an eager tail."""
        if graph_steps > 1 and n >= graph_steps:
            g = self.graph(graph_steps)
            for _ in range(n // graph_steps):
                g.replay()
            n %= graph_steps
        if n:
            self.launch(n)

    def decode_host(self, start: torch.Tensor, n: int, out: torch.Tensor | None = None,
                    graph_steps: int = 32) -> torch.Tensor:
        """Public host-buffer decode call: `start` is a (pinned) CPU int64
        tensor [5] = (token, cache_slot, t, h, w) of the first step; runs `n`
        greedy steps and returns their tokens in a (pinned) CPU int64 tensor.
        Host->device copy of the inputs and device->host copy of the tokens
        are part of the call (the reference's replay writes its inputs and
        reads the token back every step, evaluation_wrapper.py:788-791, 906-939)."""
        if out is None:
            out = torch.empty(n, dtype=torch.int64, pin_memory=True)
        if self._start_dev is None:
            self._start_dev = torch.empty(5, dtype=torch.int64, device=self.device)
        self._start_dev.copy_(start, non_blocking=True)
        # state fields token, cache_pos, rope[3] are the first five int64 words;
        # step restarts at the script end so out_tokens[step] stays in range
        st = self.state_dev.view(torch.int64)
        st[0:5].copy_(self._start_dev)
        st[5].fill_(self.script_len)
        st[AicasStepState.done_step.offset // 8].fill_(0)
        self.run(n, graph_steps)
        out.copy_(self.out_tokens[self.script_len:self.script_len + n], non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return out

    def snapshot(self):
        return self.state_dev.clone()

    def restore(self, snap):
        self.state_dev.copy_(snap)

    # ------------------------------------------------------------------ API
    def done_step(self) -> int:
        """0 while the request runs; s + 1 once step s produced the
        end-of-sequence token (reads the device state)."""
        return int(self.state_dev.view(torch.int64)[AicasStepState.done_step.offset // 8].item())

    def prefill_prompt(self, prompt, pos3=None, eos_token_id: int | None = None) -> int:
        """Prefill the whole prompt in one pass (prefill.py: library GEMMs over
        all prompt tokens, K/V written to cache slots [0, P)) and set the step
        state so the device loop continues from the first generated token,
        which is returned (its logits go to the logits ring, its id to
        out_tokens[P - 1], as with the one-token-per-launch prefill)."""
        from prefill import prefill

        tokens = torch.as_tensor(prompt, dtype=torch.int64).reshape(-1).cpu()
        P = tokens.numel()
        if P < 1 or P >= self.max_cache_len or P > self.max_steps:
            raise AicasError("prompt does not fit the cache")
        if pos3 is None:
            pos3 = torch.arange(P, dtype=torch.int64).expand(3, P)
        pos3 = torch.as_tensor(pos3, dtype=torch.int64).reshape(3, P).cpu()
        s, dev = self.shape, self.device
        with torch.cuda.device(dev):
            logits = prefill(tokens.to(dev), pos3.to(dev), self.embed, self.final_norm, self.layers, self.k_cache,
                             self.v_cache, num_heads=s.num_heads, num_kv_heads=s.num_kv_heads, head_dim=s.head_dim,
                             eps=float(s.rms_eps), inv_freq=self._inv_freq.to(dev), mrope_section=s.mrope_section)
            first = int(torch.argmax(logits))  # first index of the max, like the device argmax
            if self.logits is not None:
                self.logits[(P - 1) % self.logits_ring].copy_(logits.to(torch.float16))
            self.begin_decode(first, P, (pos3[:, -1] + 1).tolist(), eos_token_id)
        return first

    def begin_decode(self, first: int, P: int, rope, eos_token_id: int | None = None):
        """Continue a request whose prompt (P tokens) is already in the cache
        (slots [0, P)), e.g. prefilled by another implementation: `first` is
        the token its prompt produced (out_tokens[P - 1]); the next step feeds
        it at cache slot P with rope positions `rope` (3 axes).  With
        `eos_token_id`, a first token equal to it ends the request at once."""
        with torch.cuda.device(self.device):
            self.out_tokens.fill_(-1)
            self.out_tokens[P - 1] = int(first)
            # step == script_len == P: every following step decodes freely
            self._write_state(int(first), P, [int(r) for r in rope], P, P,
                              -1 if eos_token_id is None else int(eos_token_id))
            if eos_token_id is not None and int(first) == int(eos_token_id):
                self.state_dev.view(torch.int64)[AicasStepState.done_step.offset // 8].fill_(P)
        self.script_len = P

    def collect(self, P: int, max_new_tokens: int) -> torch.Tensor:
        """The request's generated tokens (CPU int64) after its steps ran: the
        first max_new_tokens from out_tokens[P - 1], cut after a device-side
        end of sequence (included)."""
        toks = self.out_tokens[P - 1:P - 1 + max_new_tokens].cpu()
        self.check_error()
        done = self.done_step()
        if done:
            toks = toks[:done - (P - 1)]
        return toks

    def generate(self, prompt, max_new_tokens: int, pos3=None, graph_steps: int = 32,
                 eos_token_id: int | None = None, prefill: str = "decode") -> torch.Tensor:
        """Greedy decode: prefill `prompt`, then max_new_tokens - 1 decode
        steps.  Returns the new tokens (CPU int64), like
        `GreedyDecodeEngine.generate` (evaluation_wrapper.py:149-315) minus the
        prompt; with `eos_token_id` the tokens end at the first generated EOS
        (included), detected on the device (the reference polls a pinned host
        copy of each token for it, evaluation_wrapper.py:317-463).
        `prefill`: "decode" runs the prompt through the decode kernel one token
        per launch; "gemm" prefills it in one pass (prefill_prompt)."""
        P = len(torch.as_tensor(prompt).reshape(-1))
        # cache slots [0, P + max_new_tokens - 1): the last token is never fed back
        if P + max_new_tokens - 1 > self.max_steps or P + max_new_tokens - 1 > self.max_cache_len:
            raise AicasError("request exceeds max_steps / max_cache_len")
        if prefill == "gemm":
            self.prefill_prompt(prompt, pos3, eos_token_id=eos_token_id)
        elif prefill == "decode":
            self.load_script(prompt, pos3, eos_token_id=eos_token_id)
            self.launch(P)
        else:
            raise ValueError(f"unknown prefill mode {prefill!r}")
        self.run(max_new_tokens - 1, graph_steps)
        return self.collect(P, max_new_tokens)

    def check_error(self):
        code = device_error(self.scratch)
        if code:
            self.reset_device_state()
            raise AicasError(f"device error {code}: {self._lib.aicas_error_string(code).decode()}")

    def reset_device_state(self):
        """After a device error: zero the scratch block and the LL vectors
        (their epochs restart with the scratch's)."""
        for t in (self.scratch, self.h, self.h_mid, self.qkv, self.attn, self.act):
            t.zero_()

    def step_logits(self, step: int) -> torch.Tensor:
        if self.logits is None:
            raise AicasError("engine built without a logits ring")
        return self.logits[step % self.logits_ring]

    # ------------------------------------------------------------------ roofline
    def algorithmic_bytes(self, cache_pos: int) -> int:
        """Bytes one step at cache slot `cache_pos` must move: all weights
        plus K/V of slots [0, cache_pos) read and the new slot written."""
        s = self.shape
        return s.weight_bytes_per_step() + s.kv_bytes_per_position() * (cache_pos + 1)


def estimate_tokens_per_second(shape: Qwen3VLTextShape, ctx: int, gbs: float) -> float:
    b = shape.weight_bytes_per_step() + shape.kv_bytes_per_position() * (ctx + 1)
    return gbs * 1e9 / b if b else math.inf
