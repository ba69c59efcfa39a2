"""Benchmark: batch-1 greedy decode of the Qwen3-VL-2B text decoder on B200.

Workload: 28-layer fp16 text decoder with seeded random
weights N(0, 0.02); KV cache prefilled from a 1024-token synthetic prefix whose
slots 16..271 are a 16x16 image grid with 3-axis MRoPE positions; then 256
greedy decode tokens, CUDA-graph captured.  One bench STEP = one such 256-token
decode request starting from the prefilled cache (the prefix stays resident,
decode slots 1024..1279 are rewritten by every step).  Weights (3.44 GB) are
streamed from HBM for every token, far above the 126 MB L2.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun, one process per GPU, each decoding its own request
(request-level data parallelism, no collective on the decode path; "weak"
scaling).  Rank 0 prints one JSON line.

`--impl reference` times the reference's CPU path instead: the CPU oracle
port (numpy fp32 restatement of the reference's HF decode step, oracle/) on
the host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "aicasgc-2026_b200"))
sys.path.insert(0, str(REPO))

PREFIX = 1024
NEW = 256
METRIC = "batch-1 decode tok/s"
UNIT = "tok/s"
FALLBACK_HBM_GBS = 6650.0


FALLBACK_BF16_TFLOPS = 1590.0


def measured_peak_gbs():
    p = REPO / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def measured_peak_tflops():
    """Dense 16-bit tensor-core peak (the driver's cuBLAS bf16 burst figure;
    fp16 runs at the same rate)."""
    p = REPO / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["bf16_tflops"]), "measured"
    except Exception:
        return FALLBACK_BF16_TFLOPS, "fallback"


def prefill_flops(shape, P: int) -> float:
    """Dense FLOPs of a P-token prefill: the projection GEMMs of every layer,
    causal attention (Q K^T and P V over the keys each query sees) and the
    LM head of the last token."""
    proj = shape.hidden * (shape.qkv_rows + shape.q_size) + shape.hidden * 3 * shape.intermediate
    attn = 2 * 2 * shape.num_heads * shape.head_dim * (P * (P + 1) // 2)
    return float(shape.num_layers * (2 * P * proj + attn) + 2 * shape.vocab * shape.hidden)


def headline_request(rank: int = 0):
    """The request one bench step decodes on `rank`: the
    1024-token prefix (seeded ids, 16x16 vision grid with 3-axis MRoPE
    positions).  Returns (prompt [PREFIX] int64, pos3 [3, PREFIX], rope_delta).
    The GPU parity test checks the same request's tokens and logits."""
    from qwen3vl_config import synthetic_prompt, vision_grid_positions

    pos3, rope_delta = vision_grid_positions(PREFIX)
    return synthetic_prompt(PREFIX, seed=1234 + rank), pos3, rope_delta


def workload_config(n_gpus: int) -> dict:
    return {
        "workload": "BASELINE config 4: Qwen3-VL-2B text decoder, 28 layers fp16, batch 1, 1024-token prefix "
                    "(16x16 vision grid, 3-axis MRoPE), 256 greedy decode tokens per step, CUDA graph",
        "model": "Qwen3-VL-2B text decoder (random init N(0,0.02))",
        "batch": 1, "prefix_len": PREFIX, "decode_tokens_per_step": NEW,
        "parallelism": f"request-dp{n_gpus}",
        "l2": "inputs larger than L2: 3.44 GB of weights streamed from HBM per token",
    }


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.idx)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sms, maxs, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sms.append(float(f[1]))
                maxs.append(float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sms) if sms else None, "sm_max_mhz": max(maxs) if maxs else None,
                "reasons": sorted(reasons), "samples": len(sms)}


# --------------------------------------------------------------------------- CPU
def cpu_oracle_decode(state16, seconds: float = 12.0, min_steps: int = 2, max_steps: int | None = None):
    """Time the CPU oracle port (numpy fp32, all host threads) decoding at
    cache slot 1024 over a synthetic KV prefix.  Returns (tok/s, steps, s)."""
    from threadpoolctl import threadpool_limits

    # all host threads, also under torchrun (which sets OMP_NUM_THREADS=1)
    threads = os.cpu_count() or 1
    with threadpool_limits(limits=threads):
        return _cpu_oracle_decode(state16, seconds, min_steps, max_steps)


def _cpu_oracle_decode(state16, seconds, min_steps, max_steps):
    import numpy as np

    from engine import hf_inv_freq
    from oracle.qwen3vl_oracle import Qwen3VLOracle
    from qwen3vl_config import QWEN3VL_2B

    cap = max_steps if max_steps is not None else 512
    o = Qwen3VLOracle(state16, QWEN3VL_2B.num_layers, mode="fp32", max_cache_len=PREFIX + cap + 2,
                      inv_freq=hf_inv_freq(QWEN3VL_2B).numpy())
    rng = np.random.default_rng(0)
    o.k_cache[:, :, :PREFIX] = rng.standard_normal(o.k_cache[:, :, :PREFIX].shape, dtype=np.float32)
    o.v_cache[:, :, :PREFIX] = rng.standard_normal(o.v_cache[:, :, :PREFIX].shape, dtype=np.float32)
    tok = 1234
    o.decode_step(tok, PREFIX, np.full((3, 1), PREFIX, np.int64))  # warm-up
    t0 = time.perf_counter()
    n = 0
    while True:
        pos = PREFIX + 1 + n
        logits = o.decode_step(tok, pos, np.full((3, 1), pos, np.int64))
        tok = int(np.argmax(logits))
        n += 1
        el = time.perf_counter() - t0
        if (n >= min_steps and el >= seconds) or n >= cap:
            break
    return n / el, n, el


def cpu_hf_decode(state16, steps: int, warmup: int):
    """The reference's own CPU path: HF's Qwen3-VL model in fp32 on the host
    cores (what `GreedyDecodeEngine` runs with ENABLE_CUDAGRAPH=0,
    evaluation_wrapper.py:149-315, 513-539), prefilled with the headline
    request's 1024-token vision-grid prefix into a StaticCache, then `steps`
    timed single-token steps through HF's forward.  Returns (tok/s, steps, s)."""
    import torch
    from transformers.cache_utils import StaticCache

    from qwen3vl_config import QWEN3VL_2B, hf_model

    torch.set_num_threads(os.cpu_count() or 1)
    m = hf_model(QWEN3VL_2B, state=state16)
    prompt, pos3, rd = headline_request(0)
    with torch.no_grad():
        cache = StaticCache(config=m.config, max_cache_len=PREFIX + warmup + steps + 1)
        out = m(input_ids=prompt.view(1, PREFIX), position_ids=pos3.view(3, 1, PREFIX), past_key_values=cache,
                use_cache=True, logits_to_keep=1)
        tok = int(out.logits[0, -1].argmax())
        t0, n = 0.0, 0
        for i in range(warmup + steps):
            if i == warmup:
                t0 = time.perf_counter()
            p = torch.full((3, 1, 1), PREFIX + i + rd, dtype=torch.long)
            out = m(input_ids=torch.tensor([[tok]]), position_ids=p, past_key_values=cache, use_cache=True)
            tok = int(out.logits[0, -1].argmax())
            n += i >= warmup
        el = time.perf_counter() - t0
    return n / el, n, el


def run_reference(args, rank: int, world: int):
    if rank != 0:
        return
    import torch

    from qwen3vl_config import QWEN3VL_2B, synthetic_state

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    st = synthetic_state(QWEN3VL_2B, seed=0, dtype=torch.float16)
    # warm-up steps then exactly K timed steps; each step = 1 decode token at ctx ~1024
    if args.ref_path == "hf":
        tps, n, el = cpu_hf_decode(st, args.steps, max(1, args.warmup))
        sample = (f"{n} decode tokens after the 1024-token vision-grid prefix, HF transformers fp32 forward with a "
                  f"StaticCache (the reference's CPU path)")
        kind = "reference"
    else:
        tps_w, _, _ = cpu_oracle_decode(st, seconds=0.0, min_steps=max(1, args.warmup),
                                        max_steps=max(1, args.warmup))
        tps, n, el = cpu_oracle_decode(st, seconds=0.0, min_steps=args.steps, max_steps=args.steps)
        sample = f"{n} decode tokens at cache slot {PREFIX}+ over a synthetic 1024-slot KV prefix (numpy fp32 port)"
        kind = "port"
    metric, config = METRIC, workload_config(world)
    if args.batch > 1:  # the reference decodes one request at a time: its batched rate is its per-token rate
        metric = f"batch-{args.batch} decode tok/s"
        config = batch_workload_config(args.batch, batch_contexts(args.batch, rank), world)
        sample += "; the reference serves one request per engine, so requests run one after another"
    line = {
        "impl": "reference", "metric": metric, "value": tps, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1000.0 * el / n, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config,
        "cpu_baseline": {"value": tps, "unit": UNIT, "cores": cores, "kind": kind, "sample": sample},
        "e2e": {"value": tps, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": ("reference arm: the reference's HF fp32 decode on the host cores" if kind == "reference" else
                 "reference arm: CPU oracle port of the reference's HF decode step") + "; a step here is one token",
    }
    print(json.dumps(line), flush=True)


def host_threads(world: int) -> int:
    """Host threads one rank uses for its setup work (weight generation): its
    share of the cores, so N ranks on one box do not oversubscribe them."""
    return max(1, (os.cpu_count() or 1) // max(1, world))


def max_over_ranks(vals, world: int):
    """Per-rank timings -> their maximum over all ranks (every rank gets it).
    Under torchrun each rank decodes its own request on its own GPU; the job
    takes as long as its slowest rank."""
    import torch
    import torch.distributed as dist

    t = torch.tensor([float(v) for v in vals], dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(x) for x in t]


def gather_ranks(row, world: int):
    """Every rank's `row` (a list of floats) -> the list of all ranks' rows
    (rank order), so rank 0 can report each GPU's own work."""
    import torch
    import torch.distributed as dist

    t = torch.tensor([float(v) for v in row], dtype=torch.float64)
    if world == 1:
        return [t.tolist()]
    out = [torch.zeros_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [x.tolist() for x in out]


def per_rank_report(rows, tokens_per_rank: int) -> list:
    """[rank, device index, timed ms, setup s] rows -> per-rank dicts with the
    rank's own tok/s (each rank's GPU decodes its own requests)."""
    return [{"rank": int(r[0]), "device": int(r[1]), "ms": r[2], "tok_s": tokens_per_rank / (r[2] / 1000.0),
             "setup_s": r[3]} for r in rows]


def job_throughput(steps: int, world: int, ms: float) -> float:
    """Whole-job tok/s: every rank decodes `steps` requests of NEW tokens in
    `ms` (the max over ranks)."""
    return steps * NEW * world / (ms / 1000.0)


# --------------------------------------------------------------------------- GPU
# DRAM bytes per algorithmic byte of decode_program_kernel, from one
# `ncu --set full` capture of the 4-layer profiling case (bench.py --layers 4;
# summarised under profiles/): (1.043188e9 + 6.631424e6) / 1043908608.  The
# per-layer shapes equal the headline model's, so the ratio carries over.
DRAM_TRAFFIC_PER_ALGORITHMIC_BYTE = 1.0056622

def run_ours(args, rank: int, world: int):
    import torch
    import torch.distributed as dist

    from engine import Qwen3VLDecodeEngine
    from qwen3vl_config import QWEN3VL_2B, synthetic_state

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("gloo", timeout=__import__("datetime").timedelta(seconds=600))

    def barrier():
        if world > 1:
            dist.barrier()

    t_setup = time.perf_counter()
    shape = QWEN3VL_2B.with_layers(args.layers)
    st = synthetic_state(shape, seed=0, dtype=torch.float16, threads=host_threads(world))
    eng = Qwen3VLDecodeEngine(st, shape, max_cache_len=PREFIX + NEW, device=dev,
                              max_steps=PREFIX + NEW + 8)
    prompt, pos3, _ = headline_request(rank)
    # prefill: one forced step per prefix token (not timed in the metric; its
    # time is the decode-kernel time to first token reported below)
    eng.load_script(prompt, pos3)
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record()
    eng.launch(PREFIX)
    p1.record()
    torch.cuda.synchronize(dev)
    ttft_decode_ms = p0.elapsed_time(p1)
    eng.check_error()
    start_state = eng.snapshot()
    first = eng.out_tokens[PREFIX - 1].item()
    graph_steps = 32
    eng.graph(graph_steps)

    def one_request():
        eng.restore(start_state)
        eng.run(NEW, graph_steps)  # 256 decode steps = 8 replays of a 32-launch graph

    setup_s = time.perf_counter() - t_setup  # weights, prefill, graph capture

    # ---- warm-up
    for _ in range(args.warmup):
        one_request()
    torch.cuda.synchronize(dev)
    eng.check_error()

    # ---- timed (device): K requests of 256 tokens
    stream = torch.cuda.current_stream(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local if "CUDA_VISIBLE_DEVICES" not in os.environ else local)
    barrier()
    torch.cuda.synchronize(dev)
    sampler.start()
    time.sleep(0.3)
    e0.record(stream)
    for _ in range(args.steps):
        one_request()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1)
    eng.check_error()
    toks = eng.out_tokens[PREFIX:PREFIX + NEW].cpu()

    # ---- timed (e2e): same requests through the host-buffer public call
    start_host = torch.tensor([first, PREFIX, *[int(x) + 1 for x in pos3[:, -1]]], dtype=torch.int64).pin_memory()
    out_host = torch.empty(NEW, dtype=torch.int64).pin_memory()
    eng.decode_host(start_host, NEW, out_host, graph_steps)
    barrier()
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    f0 = torch.cuda.Event(enable_timing=True)
    f1 = torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(args.steps):
        eng.decode_host(start_host, NEW, out_host, graph_steps)
    f1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_wall = time.perf_counter() - t0
    e2e_ms = max(f0.elapsed_time(f1), 1000 * e2e_wall)
    barrier()
    e2e_ok = bool(torch.equal(out_host, toks))

    if args.trace and rank == 0:
        write_trace_summary(eng, start_state, args.trace)

    # time to first token of the prefix with the one-pass prefill (prefill.py),
    # after a warm-up; measured last, so the launches before the timed region
    # are the same as without it (it rewrites the prefix's cache slots)
    for _ in range(2):
        eng.prefill_prompt(prompt, pos3)
    torch.cuda.synchronize(dev)
    p0.record()
    for _ in range(3):
        eng.prefill_prompt(prompt, pos3)
    p1.record()
    torch.cuda.synchronize(dev)
    ttft_gemm_ms = p0.elapsed_time(p1) / 3
    pf_flops = prefill_flops(shape, PREFIX)
    tpeak, tpeak_kind = measured_peak_tflops()

    # ---- max over ranks (and each rank's own figures: its GPU and its work)
    ranks = per_rank_report(gather_ranks([rank, dev.index, ms, setup_s], world), args.steps * NEW)
    ms, e2e_ms = max_over_ranks([ms, e2e_ms], world)
    value = job_throughput(args.steps, world, ms)
    e2e_value = job_throughput(args.steps, world, e2e_ms)
    # roofline: algorithmic bytes of the 256 launches of one request (ctx 1024..1279)
    bytes_req = sum(eng.algorithmic_bytes(PREFIX + i) for i in range(NEW))
    per_launch_s = ms / 1000.0 / (args.steps * NEW)
    achieved = bytes_req / NEW / per_launch_s / 1e9
    peak, peak_kind = measured_peak_gbs()
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16 (fp32 accumulate)", "data": "synthetic",
        "config": workload_config(world),
        "step_us_per_token": 1000.0 * ms / (args.steps * NEW),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": peak_kind,
                     "traffic": DRAM_TRAFFIC_PER_ALGORITHMIC_BYTE * bytes_req / NEW,
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one 4-layer "
                                       "launch (1.0432 GB + 6.6 MB vs 1.0439 GB algorithmic), scaled to this "
                                       "launch by algorithmic bytes",
                     "kernel": "decode_program_kernel (one launch per token)",
                     "algorithmic_bytes_per_launch": bytes_req / NEW},
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": 40, "d2h_bytes_per_step": 8 * NEW,
                "tokens_match_device_run": e2e_ok},
        "gpu_launches": args.steps * NEW,
        "per_rank": ranks,
        "ttft": {"prefix_tokens": PREFIX, "one_pass_prefill_ms": ttft_gemm_ms,
                 "decode_kernel_prefill_ms": ttft_decode_ms,
                 "roofline": {"bound": "tensor", "flops": pf_flops,
                              "achieved_tflops": pf_flops / (ttft_gemm_ms * 1e-3) / 1e12, "peak": tpeak,
                              "peak_kind": tpeak_kind, "unit": "TFLOP/s",
                              "frac": pf_flops / (ttft_gemm_ms * 1e-3) / 1e12 / tpeak},
                 "note": "first token of the 1024-token prefix (prefill_native: hand-written prefill kernels "
                         "between cuBLAS fp16 GEMMs); outside the decode metric"},
        "clocks": clocks,
    }
    if args.layers != QWEN3VL_2B.num_layers:
        line["config"]["workload"] = f"profiling case ({args.layers} layers), not the headline workload"
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.layers == QWEN3VL_2B.num_layers:
        tps, n, el = cpu_oracle_decode(st, seconds=args.cpu_seconds)
        line["cpu_baseline"] = {"value": tps, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
                                "sample": f"{n} decode tokens ({el:.1f} s) at cache slot {PREFIX}+ over a synthetic "
                                          f"KV prefix, numpy fp32 oracle port, all host threads"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


BATCH_NEW = 512  # decode steps per stream per bench step (config 5)


def batch_workload_config(batch: int, ctx: list, n_gpus: int) -> dict:
    return {"workload": f"BASELINE config 5 per GPU: Qwen3-VL-2B text decoder, 28 layers fp16, {batch} ragged "
                        f"requests (contexts {ctx}, U[512, 4096] seeded), {BATCH_NEW} greedy decode steps "
                        f"per request per bench step, one batched launch per step, CUDA graph",
            "model": "Qwen3-VL-2B text decoder (random init N(0,0.02))", "batch": batch,
            "contexts": ctx, "decode_steps_per_request": BATCH_NEW, "parallelism": f"request-dp{n_gpus}",
            "l2": "inputs larger than L2: 3.44 GB of weights + the requests' KV streamed per step"}
# DRAM bytes per algorithmic byte of decode_batch_kernel, from one `ncu --set
# full` capture of the 2-layer batch-8 profiling case (bench.py --batch 8
# --layers 2; summarised under profiles/): (983.693568e6 + 15.259648e6) /
# 981263360 (reads 0.2 % above the algorithmic bytes, the rest writes).
BATCH_DRAM_TRAFFIC_PER_ALGORITHMIC_BYTE = 1.0180276
BATCH_CTX = (512, 4096)  # per-stream context lengths, uniform, seeded


def batch_contexts(batch: int, rank: int) -> list[int]:
    import numpy as np

    rng = np.random.default_rng(5 + rank)
    return [int(x) for x in rng.integers(BATCH_CTX[0], BATCH_CTX[1] + 1, size=batch)]


def run_batch(args, rank: int, world: int):
    """BASELINE config 5 on each GPU: `--batch` ragged requests decoded
    together by the batched kernel (one launch per step for all streams).
    One bench STEP = BATCH_NEW batched decode steps from the prefilled
    caches (B x BATCH_NEW tokens)."""
    import torch
    import torch.distributed as dist

    from batch_engine import Qwen3VLBatchDecodeEngine
    from qwen3vl_config import QWEN3VL_2B, synthetic_prompt, synthetic_state, vision_grid_positions

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("gloo", timeout=__import__("datetime").timedelta(seconds=600))

    def barrier():
        if world > 1:
            dist.barrier()

    t_setup = time.perf_counter()
    B = args.batch
    ctx = batch_contexts(B, rank)
    shape = QWEN3VL_2B.with_layers(args.layers)
    st = synthetic_state(shape, seed=0, dtype=torch.float16, threads=host_threads(world))
    lmax = max(ctx) + BATCH_NEW + 8
    eng = Qwen3VLBatchDecodeEngine(st, shape, max_batch=B, max_cache_len=lmax, device=dev, max_steps=lmax)
    firsts, pos_next = [], []
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    p0.record()
    for b, P in enumerate(ctx):
        pos3, _ = vision_grid_positions(P)
        firsts.append(eng.add_request(b, synthetic_prompt(P, seed=2000 + 17 * rank + b), pos3))
        pos_next.append([int(x) + 1 for x in pos3[:, -1]])
    p1.record()
    torch.cuda.synchronize(dev)
    prefill_ms = p0.elapsed_time(p1)
    start_state = eng.state_dev.clone()
    graph_steps = 32
    eng.graph(graph_steps)

    def one_step():
        eng.state_dev.copy_(start_state)
        eng.run(BATCH_NEW, graph_steps)

    setup_s = time.perf_counter() - t_setup

    for _ in range(args.warmup):
        one_step()
    torch.cuda.synchronize(dev)
    eng.check_error()
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    barrier()
    torch.cuda.synchronize(dev)
    sampler.start()
    time.sleep(0.3)
    e0.record(stream)
    for _ in range(args.steps):
        one_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1)
    eng.check_error()
    toks = torch.stack([eng.out_tokens[b, P:P + BATCH_NEW] for b, P in enumerate(ctx)]).cpu()

    # e2e: the same steps through the host-buffer call (inputs H2D, tokens D2H)
    start_host = torch.tensor([[f, P, *pn] for f, P, pn in zip(firsts, ctx, pos_next)],
                              dtype=torch.int64).pin_memory()
    out_host = torch.empty((B, BATCH_NEW), dtype=torch.int64).pin_memory()
    eng.decode_host(start_host, BATCH_NEW, out_host, graph_steps)
    barrier()
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(args.steps):
        eng.decode_host(start_host, BATCH_NEW, out_host, graph_steps)
    f1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = max(f0.elapsed_time(f1), 1000 * (time.perf_counter() - t0))
    barrier()
    e2e_ok = bool(torch.equal(out_host, toks))

    ranks = per_rank_report(gather_ranks([rank, dev.index, ms, setup_s], world), args.steps * B * BATCH_NEW)
    ms, e2e_ms = max_over_ranks([ms, e2e_ms], world)
    tok_per_step = B * BATCH_NEW
    value = args.steps * tok_per_step * world / (ms / 1000.0)
    e2e_value = args.steps * tok_per_step * world / (e2e_ms / 1000.0)
    bytes_step = sum(eng.algorithmic_bytes([P + i for P in ctx]) for i in range(BATCH_NEW))
    per_launch_s = ms / 1000.0 / (args.steps * BATCH_NEW)
    achieved = bytes_step / BATCH_NEW / per_launch_s / 1e9
    peak, peak_kind = measured_peak_gbs()
    line = {
        "metric": f"batch-{B} decode tok/s", "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16 (fp32 accumulate)", "data": "synthetic",
        "config": batch_workload_config(B, ctx, world),
        "us_per_batched_step": 1000.0 * ms / (args.steps * BATCH_NEW),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_kind": peak_kind,
                     "traffic": BATCH_DRAM_TRAFFIC_PER_ALGORITHMIC_BYTE * bytes_step / BATCH_NEW,
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one 2-layer batch-8 "
                                       "launch (983.7 MB + 15.3 MB vs 981.3 MB algorithmic), scaled to this "
                                       "launch by algorithmic bytes",
                     "kernel": "decode_batch_kernel (one launch per batched step)",
                     "algorithmic_bytes_per_launch": bytes_step / BATCH_NEW},
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": 40 * B,
                "d2h_bytes_per_step": 8 * B * BATCH_NEW, "tokens_match_device_run": e2e_ok},
        "gpu_launches": args.steps * BATCH_NEW,
        "per_rank": ranks,
        "prefill_ms_all_requests": prefill_ms,
        "clocks": clocks,
    }
    if args.layers != QWEN3VL_2B.num_layers:
        line["config"]["workload"] = f"profiling case ({args.layers} layers), not the config-5 workload"
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


# ---------------------------------------------------------------- op benchmarks
GEMV_SHAPES = [("qkv", 4096, 2048), ("o_proj", 2048, 2048), ("gate_up", 12288, 2048), ("down", 2048, 6144),
               ("lm_head_argmax", 151936, 2048)]
ATTN_LENGTHS = [128, 512, 1024, 2048, 4096, 8192]
OP_COPIES = 28  # distinct weight / KV copies visited round-robin: the working set exceeds L2


def _cpu_op_baseline(fn, seconds: float):
    """Median seconds per call of `fn` on the host (all threads), at least 3
    calls and about `seconds` of work."""
    from threadpoolctl import threadpool_limits

    with threadpool_limits(limits=os.cpu_count() or 1):
        fn()
        ts = []
        t_end = time.perf_counter() + seconds
        while len(ts) < 3 or time.perf_counter() < t_end:
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
            if len(ts) >= 200:
                break
    return statistics.median(ts), len(ts)


def _time_graph(torch, calls, reps: int, warmup: int, dev):
    """Capture `calls` (a list of zero-argument launches) in one CUDA graph,
    replay it `warmup` + `reps` times; returns device us per call (CUDA
    events on the capturing stream)."""
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        for c in calls:  # eager warm-up outside capture
            c()
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for c in calls:
                c()
        for _ in range(warmup):
            g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        stream.synchronize()
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
        stream.synchronize()
    return 1000.0 * e0.elapsed_time(e1) / (reps * len(calls))


def run_op(args, rank: int, world: int):
    """BASELINE configs 2 (decode GEMV shapes, fused GEMV entries) and 3
    (decode attention alone), and the q/k norm + rotary + KV write small op:
    one JSON line per shape / valid length, each op called through
    the C ABI (the reference-facing entry points), one call per distinct
    weight or KV copy so the working set exceeds L2, as one CUDA graph."""
    if rank != 0:
        return
    import ctypes

    import numpy as np
    import torch

    import _native
    from oracle.qwen3vl_oracle import attention_reference, gemv_reference

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    L = _native.lib()
    peak, peak_kind = measured_peak_gbs()
    cores = os.cpu_count()
    scratch = torch.zeros(_native.scratch_bytes(), dtype=torch.uint8, device=dev)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    g = torch.Generator(device=dev).manual_seed(7)  # inputs made on the device (17 GB of lm_head copies)
    lines = []

    def emit(name, shape, us, algo_bytes, cpu_s, cpu_n, cpu_sample, extra):
        achieved = algo_bytes / (us * 1e-6) / 1e9
        line = {"metric": f"decode {args.op} op us per call", "op": name, "shape": shape, "value": us,
                "unit": "us", "higher_is_better": False, "n_gpus": 1, "dtype": "f16 (fp32 accumulate)",
                "data": "synthetic",
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                             "frac": achieved / peak, "peak_kind": peak_kind, "algorithmic_bytes": algo_bytes},
                "cpu_baseline": {"value": cpu_s * 1e6, "unit": "us", "cores": cores, "kind": "port",
                                 "sample": f"{cpu_n} calls, {cpu_sample}"},
                "config": {"workload": ("BASELINE config 2: decode GEMV, fp16 weights N(0,0.02), x N(0,1)"
                                        if args.op == "gemv" else
                                        "decode small op: q/k RMSNorm + rotary + static-KV write of one token, "
                                        "16 query / 8 KV heads, 8192-slot cache" if args.op == "small" else
                                        "BASELINE config 3: decode attention, q [1,16,128], K/V [8,L,128] "
                                        "N(0,1) in an 8192-slot cache, scale 1/sqrt(128)"),
                           "copies": OP_COPIES, "l2": "one distinct weight / KV copy per call, "
                                                       f"{OP_COPIES} copies round-robin (working set > L2)"},
                **extra}
        lines.append(line)
        print(json.dumps(line), flush=True)

    if args.op == "gemv":
        for name, n, k in GEMV_SHAPES:
            ws = [(torch.randn((n, k), generator=g, device=dev) * 0.02).half() for _ in range(OP_COPIES)]
            x = torch.randn(k, generator=g, device=dev).half()
            y = torch.empty(n, dtype=torch.float16, device=dev)
            tok = torch.empty(1, dtype=torch.int64, device=dev)
            stream_of = lambda: ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)  # noqa: E731
            if name == "lm_head_argmax":
                calls = [lambda w=w: _native.check(L.aicas_lm_head_argmax_f16(
                    p(x), None, p(w), p(y), p(tok), n, k, 0.0, p(scratch), stream_of()), "lm_head")
                    for w in ws]
            else:
                calls = [lambda w=w: _native.check(L.aicas_gemv_f16(
                    p(x), p(w), None, p(y), n, k, p(scratch), stream_of()), "gemv") for w in ws]
            us = _time_graph(torch, calls, reps=args.steps, warmup=args.warmup, dev=dev)
            w0, x0 = ws[-1].float().cpu().numpy(), x.float().cpu().numpy()
            ok = bool(np.allclose(y.float().cpu().numpy(), gemv_reference(w0, x0), atol=2e-3, rtol=2e-3))
            if name == "lm_head_argmax":
                ok = ok and int(tok.item()) == int(np.argmax(gemv_reference(w0, x0)))
            cpu_s, cpu_n = _cpu_op_baseline(lambda: gemv_reference(w0, x0), args.cpu_seconds / 5)
            emit(name, [n, k], us, n * k * 2 + k * 2 + n * 2, cpu_s, cpu_n,
                 "numpy fp32 W x (the oracle's restatement of F.linear), all host threads",
                 {"matches_oracle": ok})
            del ws
            torch.cuda.empty_cache()
        # the fused entry points of the drop-in (cuda_decode_gemv.fused_rmsnorm_qkv_half and
        # fused_post_attn_mlp_softsync_half): RMSNorm + QKV, and add + RMSNorm + gate_up + SiLU*up
        # + down + residual (two launches)
        from oracle.qwen3vl_oracle import post_attn_mlp_reference, rms_norm

        hid, inter = 2048, 6144
        stream_of = lambda: ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)  # noqa: E731
        x = torch.randn(hid, generator=g, device=dev).half()
        a2 = torch.randn(hid, generator=g, device=dev).half()
        nw = (1 + 0.1 * torch.randn(hid, generator=g, device=dev)).half()
        wq = [(torch.randn((4096, hid), generator=g, device=dev) * 0.02).half() for _ in range(OP_COPIES)]
        y = torch.empty(4096, dtype=torch.float16, device=dev)
        calls = [lambda w=w: _native.check(L.aicas_rmsnorm_qkv_f16(
            p(x), p(nw), p(w), None, p(y), 4096, hid, 1e-6, p(scratch), stream_of()), "rmsnorm_qkv") for w in wq]
        us = _time_graph(torch, calls, reps=args.steps, warmup=args.warmup, dev=dev)
        xn = rms_norm(x.float().cpu().numpy(), nw.float().cpu().numpy(), 1e-6)
        w0 = wq[-1].float().cpu().numpy()
        ok = bool(np.allclose(y.float().cpu().numpy(), gemv_reference(w0, xn), atol=2e-3, rtol=2e-3))
        cpu_s, cpu_n = _cpu_op_baseline(lambda: gemv_reference(w0, rms_norm(x.float().cpu().numpy(),
                                                                            nw.float().cpu().numpy(), 1e-6)),
                                        args.cpu_seconds / 5)
        emit("rmsnorm_qkv", [4096, hid], us, 4096 * hid * 2 + 2 * hid * 2 + 4096 * 2, cpu_s, cpu_n,
             "numpy fp32 RMSNorm then W x (the oracle's restatement), all host threads", {"matches_oracle": ok})
        del wq
        torch.cuda.empty_cache()
        wgu = [(torch.randn((2 * inter, hid), generator=g, device=dev) * 0.02).half() for _ in range(OP_COPIES)]
        wd = [(torch.randn((hid, inter), generator=g, device=dev) * 0.02).half() for _ in range(OP_COPIES)]
        act = torch.empty(inter, dtype=torch.float16, device=dev)
        out = torch.empty(hid, dtype=torch.float16, device=dev)
        calls = [lambda u=u, dw=dw: _native.check(L.aicas_post_attn_mlp_f16(
            p(x), p(a2), p(nw), p(u), p(dw), None, p(act), p(out), hid, inter, 1e-6, p(scratch), stream_of()),
            "post_attn_mlp") for u, dw in zip(wgu, wd)]
        us = _time_graph(torch, calls, reps=args.steps, warmup=args.warmup, dev=dev)
        f = lambda t: t.float().cpu().numpy()  # noqa: E731
        args_ref = (f(x), f(a2), f(nw), f(wgu[-1]), f(wd[-1]))
        ract, rout = post_attn_mlp_reference(*args_ref)
        ok = bool(np.allclose(f(act), ract, atol=2e-3, rtol=2e-3)
                  and np.abs(f(out) - rout).max() <= 4e-3 * max(1.0, float(np.abs(rout).max())))
        cpu_s, cpu_n = _cpu_op_baseline(lambda: post_attn_mlp_reference(*args_ref), args.cpu_seconds / 5)
        emit("post_attn_mlp", [2 * inter, hid, hid, inter], us,
             (2 * inter * hid + hid * inter) * 2 + 4 * hid * 2 + 2 * inter * 2, cpu_s, cpu_n,
             "numpy fp32 add + RMSNorm + gate_up + SiLU*up + down + residual (the oracle's restatement), "
             "all host threads", {"matches_oracle": ok, "launches_per_call": 2})
        del wgu, wd
        torch.cuda.empty_cache()
    elif args.op == "small":
        # cuda_decode_small_ops.fused_q_rope_kv_cache_update: q/k RMSNorm + rotary + the static-KV write of
        # one token (16 query heads, 8 KV heads) into a distinct 8192-slot cache per call
        from oracle.qwen3vl_oracle import rms_norm, rope

        lmax = 8192
        q = torch.randn(16 * 128, generator=g, device=dev).half()
        kk = torch.randn(8 * 128, generator=g, device=dev).half()
        vv = torch.randn(8 * 128, generator=g, device=dev).half()
        qw = (1 + 0.1 * torch.randn(128, generator=g, device=dev)).half()
        kw = (1 + 0.1 * torch.randn(128, generator=g, device=dev)).half()
        ang = torch.arange(128, dtype=torch.float32, device=dev) * 0.37
        cos, sin = torch.cos(ang).half(), torch.sin(ang).half()
        kcs = [torch.zeros((8, lmax, 128), dtype=torch.float16, device=dev) for _ in range(OP_COPIES)]
        vcs = [torch.zeros((8, lmax, 128), dtype=torch.float16, device=dev) for _ in range(OP_COPIES)]
        qo = torch.empty_like(q)
        pos = torch.tensor([4095], dtype=torch.int64, device=dev)
        stream_of = lambda: ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)  # noqa: E731
        calls = [lambda kc=kc, vc=vc: _native.check(L.aicas_qk_norm_mrope_kvwrite_f16(
            p(q), p(kk), p(vv), p(qw), p(kw), p(cos), p(sin), p(qo), p(kc), p(vc), p(pos), 1e-6, 16, 8, lmax,
            stream_of()), "q_rope_kv") for kc, vc in zip(kcs, vcs)]
        us = _time_graph(torch, calls, reps=args.steps, warmup=args.warmup, dev=dev)
        f = lambda t: t.float().cpu().numpy()  # noqa: E731
        c, s_ = f(cos).reshape(1, 128), f(sin).reshape(1, 128)
        ref = lambda: (rope(rms_norm(f(q).reshape(1, 16, 128), f(qw), 1e-6), c, s_),  # noqa: E731
                       rope(rms_norm(f(kk).reshape(1, 8, 128), f(kw), 1e-6), c, s_))
        rq, rk = ref()
        ok = bool(np.abs(f(qo).reshape(1, 16, 128) - rq).max() <= 2e-3
                  and np.abs(f(kcs[-1][:, 4095]) - rk[0]).max() <= 2e-3
                  and np.array_equal(f(vcs[-1][:, 4095]), f(vv).reshape(8, 128)))
        cpu_s, cpu_n = _cpu_op_baseline(ref, args.cpu_seconds / 5)
        # bytes: q, k, v in; q out; the k / v slot rows written; norm weights and cos / sin
        emit("q_rope_kv_update", [16, 8, 128], us, (16 * 128 * 2 + 8 * 128 * 2) * 2 + 2 * 128 * 2 * 2, cpu_s,
             cpu_n, "numpy fp32 q/k RMSNorm + rotary (the oracle's restatement), all host threads",
             {"matches_oracle": ok, "bound_note": "12 KB per call: launch- and latency-bound, not HBM-bound"})
    else:
        lmax = 8192
        scale = 128 ** -0.5
        q = torch.randn(16 * 128, generator=g, device=dev).half()
        ks = [torch.randn((8, lmax, 128), generator=g, device=dev).half() for _ in range(OP_COPIES)]
        vs = [torch.randn((8, lmax, 128), generator=g, device=dev).half() for _ in range(OP_COPIES)]
        out = torch.empty(16 * 128, dtype=torch.float16, device=dev)
        for Lv in ATTN_LENGTHS:
            pos = torch.tensor([Lv - 1], dtype=torch.int64, device=dev)
            stream_of = lambda: ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)  # noqa: E731
            calls = [lambda kc=kc, vc=vc: _native.check(L.aicas_decode_attn_splitkv_f16(
                p(q), p(kc), p(vc), p(pos), scale, p(out), 16, 8, lmax, p(scratch), stream_of()), "attention")
                for kc, vc in zip(ks, vs)]
            us = _time_graph(torch, calls, reps=args.steps, warmup=args.warmup, dev=dev)
            q0 = q.view(16, 128).float().cpu().numpy()
            k0 = ks[-1][:, :Lv].float().cpu().numpy()
            v0 = vs[-1][:, :Lv].float().cpu().numpy()
            ref = attention_reference(q0, k0, v0, Lv, scale)
            ok = bool(np.abs(out.view(16, 128).float().cpu().numpy() - ref).max() <= 2e-3)
            cpu_s, cpu_n = _cpu_op_baseline(lambda: attention_reference(q0, k0, v0, Lv, scale),
                                            args.cpu_seconds / 6)
            emit(f"attention_L{Lv}", [16, 8, Lv, 128], us, 4096 * Lv + 2 * 16 * 128 * 2, cpu_s, cpu_n,
                 "numpy fp32 restatement of the reference's _hf_repeat_kv_attention, all host threads",
                 {"valid_len": Lv, "matches_oracle": ok})
    if args.op_out:
        Path(args.op_out).write_text("\n".join(json.dumps(x) for x in lines) + "\n")


def run_prefill_op(args, rank: int, world: int):
    """Time to first token of the headline request's 1024-token prefix (16x16
    vision grid) through the native one-pass prefill (engine.prefill_prompt ->
    prefill_native), 28 layers: ms per prefill (CUDA events), its dense-FLOP
    roofline against the measured 16-bit tensor peak, and the CPU oracle's
    prefill of the same prompt as the baseline."""
    if rank != 0:
        return
    import numpy as np
    import torch

    from engine import Qwen3VLDecodeEngine, hf_inv_freq
    from oracle.qwen3vl_oracle import Qwen3VLOracle
    from qwen3vl_config import QWEN3VL_2B, synthetic_state

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    shape = QWEN3VL_2B.with_layers(args.layers)
    st = synthetic_state(shape, seed=0, dtype=torch.float16)
    eng = Qwen3VLDecodeEngine(st, shape, max_cache_len=PREFIX + NEW, device=dev, max_steps=PREFIX + NEW + 8)
    prompt, pos3, _ = headline_request(0)
    for _ in range(args.warmup):
        eng.prefill_prompt(prompt, pos3)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        first = eng.prefill_prompt(prompt, pos3)
    e1.record()
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / args.steps
    flops = prefill_flops(shape, PREFIX)
    tpeak, tpeak_kind = measured_peak_tflops()
    achieved = flops / (ms * 1e-3) / 1e12
    line = {"metric": "prefill time to first token", "value": ms, "unit": "ms", "higher_is_better": False,
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "dtype": "f16 (fp32 accumulate)",
            "data": "synthetic", "first_token": first,
            "config": {"workload": f"BASELINE config 4 prefix: {PREFIX}-token prompt (16x16 vision grid, 3-axis "
                                   f"MRoPE), {shape.num_layers} layers, one-pass native prefill"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": tpeak, "unit": "TFLOP/s",
                         "frac": achieved / tpeak, "peak_kind": tpeak_kind, "flops": flops}}
    if not args.no_cpu_baseline and args.layers == QWEN3VL_2B.num_layers:
        from threadpoolctl import threadpool_limits

        with threadpool_limits(limits=os.cpu_count() or 1):
            o = Qwen3VLOracle(st, shape.num_layers, mode="fp32", max_cache_len=PREFIX + 8,
                              inv_freq=hf_inv_freq(shape).numpy())
            t0 = time.perf_counter()
            logits = o.prefill(prompt.numpy(), pos3.numpy())
            el = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": 1000 * el, "unit": "ms", "cores": os.cpu_count(), "kind": "port",
                                "sample": "one prefill of the same prompt, numpy fp32 oracle port, all host threads",
                                "first_token": int(np.argmax(logits))}
    print(json.dumps(line), flush=True)


def run_ops_path(args, rank: int, world: int):
    """The headline request decoded through the drop-in
    ops instead of the persistent step kernel: per layer the five calls the
    reference's OptimizedDecoderLayer decode branch makes (fused RMSNorm +
    QKV, q/k norm + rotary + KV write, split-KV attention, o_proj GEMV, the
    post-attention MLP), then the fused lm_head + argmax, the next token's
    embedding row and the rotary cos/sin computed on the device: one CUDA
    graph per decode step (about 6 launches per layer), 256 steps per bench
    step.  This is what a caller of the reference's per-op interface gets
    from these kernels; the headline path runs the same math as one launch
    per token.  Tokens are compared with the step kernel's for the same
    request.  One GPU, rank 0."""
    if rank != 0:
        return
    import torch

    import _ops
    from engine import Qwen3VLDecodeEngine, hf_inv_freq
    from qwen3vl_config import QWEN3VL_2B, synthetic_state

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    shape = QWEN3VL_2B.with_layers(args.layers)
    st = synthetic_state(shape, seed=0, dtype=torch.float16, threads=host_threads(world))
    eng = Qwen3VLDecodeEngine(st, shape, max_cache_len=PREFIX + NEW, device=dev, max_steps=PREFIX + NEW + 8,
                              logits_ring=PREFIX + NEW)
    prompt, pos3, _ = headline_request(rank)
    first = eng.prefill_prompt(prompt, pos3)
    start_state = eng.snapshot()
    eng.run(NEW, 32)
    torch.cuda.synchronize(dev)
    eng.check_error()
    ref_toks = eng.out_tokens[PREFIX:PREFIX + NEW].cpu()

    s = shape
    eps, scale = float(s.rms_eps), s.head_dim ** -0.5
    qs, ks = s.num_heads * s.head_dim, s.num_kv_heads * s.head_dim
    f16 = dict(dtype=torch.float16, device=dev)
    i64 = dict(dtype=torch.int64, device=dev)
    inv = hf_inv_freq(s).to(device=dev, dtype=torch.float32)
    half = s.head_dim // 2
    axis = torch.zeros(half, **i64)  # interleaved MRoPE: frequency i takes axis 1 / 2 / 0
    for i in range(half):
        if i % 3 == 1 and i < 3 * s.mrope_section[1]:
            axis[i] = 1
        elif i % 3 == 2 and i < 3 * s.mrope_section[2]:
            axis[i] = 2
    rope0 = torch.tensor([int(x) + 1 for x in pos3[:, -1]], **i64)
    tok, pos, rope = torch.tensor([first], **i64), torch.tensor([PREFIX], **i64), rope0.clone()
    out_tok = torch.zeros(NEW, **i64)
    qkv, q_rot, attn, o = (torch.empty(n, **f16) for n in (qs + 2 * ks, qs, qs, s.hidden))
    act = torch.empty(s.intermediate, **f16)
    hb = [torch.empty(s.hidden, **f16) for _ in range(2)]

    def step():
        h = torch.index_select(eng.embed, 0, tok).view(-1)
        ang = inv * torch.index_select(rope, 0, axis).to(torch.float32)
        emb = torch.cat([ang, ang])
        cos, sin = emb.cos().to(torch.float16), emb.sin().to(torch.float16)
        for li, lw in enumerate(eng.layers):
            _ops.gemv(h, lw["qkv"], norm_w=lw["ln1"], eps=eps, out=qkv)
            kc, vc = eng.k_cache[li][0], eng.v_cache[li][0]
            _ops.qk_norm_rope_kvwrite(qkv[:qs], qkv[qs:qs + ks], qkv[qs + ks:], lw["qn"], lw["kn"], cos, sin, kc, vc,
                                      pos, eps, q_out=q_rot)
            _ops.decode_attention(q_rot, kc, vc, pos, scale, out=attn)
            _ops.gemv(attn, lw["o"], out=o)
            hn = hb[li % 2]
            _ops.post_attn_mlp(h, o, lw["ln2"], lw["gate_up"], lw["down_rm"], eps=eps, act_out=act, out=hn)
            h = hn
        _ops.lm_head_argmax(h, eng.embed, norm_w=eng.final_norm, eps=eps, token_out=tok, want_logits=False)
        out_tok.index_copy_(0, pos - PREFIX, tok)
        pos.add_(1)
        rope.add_(1)

    def reset():
        eng.restore(start_state)
        tok.fill_(first)
        pos.fill_(PREFIX)
        rope.copy_(rope0)

    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        reset()
        step()  # eager warm-up outside capture
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step()
        reset()
        for _ in range(NEW):
            g.replay()
        stream.synchronize()
        eng.check_error()
        toks = out_tok.cpu()
        same = int((toks == ref_toks).cumprod(0).sum())  # steps equal to the step kernel's, up to the first difference
        gap = None
        if same < NEW:  # the step kernel's top-2 logit gap where the two paths first differ
            top = eng.step_logits(PREFIX + same).float().topk(2).values
            gap = float(top[0] - top[1])
        for _ in range(args.warmup):
            reset()
            for _ in range(NEW):
                g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        stream.synchronize()
        ms = 0.0
        for _ in range(args.steps):
            reset()
            e0.record(stream)
            for _ in range(NEW):
                g.replay()
            e1.record(stream)
            stream.synchronize()
            ms += e0.elapsed_time(e1)
    us_tok = 1000.0 * ms / (args.steps * NEW)
    line = {"metric": METRIC, "path": "drop-in ops: the five per-layer op calls of the reference's decoder layer + "
                                      "lm_head/argmax, one CUDA graph per token",
            "value": 1e6 / us_tok, "unit": UNIT, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "us_per_token": us_tok, "higher_is_better": True, "dtype": "f16 (fp32 accumulate)", "data": "synthetic",
            "config": workload_config(1), "tokens_equal_to_step_kernel": f"{same} of {NEW}",
            "top2_gap_at_first_difference": gap}
    print(json.dumps(line), flush=True)


def write_trace_summary(eng, start_state, path):
    """One traced decode step at cache slot 1024.  Per phase kind (summed
    over layers, averaged over CTAs): time waiting for inputs, time from
    inputs to phase end, tile-wait time, producer slot-wait time, tiles per
    CTA; plus the step's wall time."""
    import torch

    eng.restore(start_state)
    tr = eng.launch_traced().double()  # [cta, phase, 8]
    names = eng.phase_names()
    t0 = tr[:, 0, 0].min()
    start, ready, end = tr[:, :, 0] - t0, tr[:, :, 1] - t0, tr[:, :, 2] - t0
    kinds = {}
    for i, nm in enumerate(names):
        k = nm.split(".")[-1]
        e = kinds.setdefault(k, {"n": 0, "input_wait_us": 0.0, "work_us": 0.0, "tile_wait_us": 0.0,
                                 "producer_slot_wait_us": 0.0, "tiles_per_cta": 0.0, "span_us": 0.0})
        e["n"] += 1
        e["input_wait_us"] += float((ready[:, i] - start[:, i]).mean()) / 1e3
        e["work_us"] += float((end[:, i] - ready[:, i]).mean()) / 1e3
        e["tile_wait_us"] += float(tr[:, i, 3].mean()) / 1e3
        e["producer_slot_wait_us"] += float(tr[:, i, 4].mean()) / 1e3
        e["tiles_per_cta"] += float(tr[:, i, 5].mean())
        e["span_us"] += float(end[:, i].max() - start[:, i].min()) / 1e3
    total = float(end.max() - start.min()) / 1e3
    summary = {"step_us": total, "by_kind_total": kinds}
    import numpy as np

    np.save(str(Path(path).with_suffix(".npy")), tr.numpy().astype(np.int64))
    Path(path).parent.mkdir(parents=True, exist_ok=True)
    Path(path).write_text(json.dumps(summary, indent=1))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ref-path", choices=["port", "hf"], default="port",
                    help="--impl reference: time the numpy oracle port (default) or HF transformers' own fp32 "
                         "forward (the reference's CPU path; needs transformers)")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--trace", default="", help="write a per-phase timeline summary (JSON) to this path")
    ap.add_argument("--batch", type=int, default=1,
                    help="requests per GPU: 1 = BASELINE config 4 (the headline); 2..8 = config 5's batched "
                         "decode of ragged requests (contexts U[512, 4096], 512 decode steps each)")
    ap.add_argument("--layers", type=int, default=28,
                    help="profiling case only: a smaller model (the headline is 28 layers)")
    ap.add_argument("--op", choices=["gemv", "attention", "small", "prefill"], default=None,
                    help="per-op benchmark instead of the decode step: BASELINE config 2 (the five decode GEMV "
                         "shapes and the fused RMSNorm+QKV / post-attention MLP entries), config 3 (decode "
                         "attention at valid lengths 128..8192; --steps = graph replays of one call per copy), "
                         "the q/k norm + rotary + KV write small op, or the headline prefix's one-pass prefill "
                         "(TTFT)")
    ap.add_argument("--op-out", default="", help="also write the op benchmark's JSON lines to this file")
    ap.add_argument("--path", choices=["step", "ops"], default="step",
                    help="ops: decode the headline request through the drop-in per-op entry points (one CUDA graph "
                         "per token) instead of the persistent step kernel; one GPU")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.op == "prefill":
        run_prefill_op(args, rank, world)
    elif args.op:
        run_op(args, rank, world)
    elif args.path == "ops":
        run_ops_path(args, rank, world)
    elif args.impl == "reference":
        run_reference(args, rank, world)
    elif args.batch > 1:
        run_batch(args, rank, world)
    else:
        run_ours(args, rank, world)


if __name__ == "__main__":
    main()
