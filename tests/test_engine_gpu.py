"""GPU parity of the whole decode step (the persistent phase-program kernel).

* 2-layer model vs the reference's own golden outputs (fp32 HF through the
  reference's `GreedyDecodeEngine`): identical greedy tokens, logits within
  5e-2 (fp16 engine vs fp32 reference).
* 2-layer and full 28-layer models vs the fp16 oracle, teacher-forced on the
  engine's own trajectory: logits within tolerance at every step, and every
  token equal to the oracle's argmax unless the oracle's top-2 gap is below
  the tolerance (a genuine near-tie that fp32 summation order may break
  either way).

Tolerance.  2 layers: max |d logit| <= 2e-2 at every step.  28 layers: the
test decodes the benchmarked request itself (bench.py's `headline_request`:
1024-token prefix with a vision grid, then the first token and 256 decode
steps, 257 tokens in all) against the fp16 oracle with float64 sums
(`accumulate="f64"`: HF's fp16 rounding points, exact matmul and reduction
sums), and measures in the same run the noise floor of fp32 summation: the
same oracle with float32 sums against the float64 one.  Any fp32-summing
implementation flips an occasional fp16 rounding where its sum lands next to
a rounding boundary; over 28 residual layers those flips move the logits by
up to ~0.02, for two correct CPU implementations as much as for the GPU
(measured over 40 of these steps on the CPU: float32 vs float64 sums max
0.0225, median 0.0176 per step; the GPU against float64 sums over all 257:
max 0.0226, median 0.0176).  HF's own fp16 model run on a B200 (cuBLAS +
SDPA) on the same tokens is much further from the exact sums: median 0.32,
max 0.53 per step.  The 28-layer bounds are therefore: mean |d| <= 5e-3 at every
step, median over steps of the per-step max <= 2e-2, and the worst step
within max(2e-2, 1.15 x the floor's worst step); each step's token equals
the oracle's argmax unless the oracle's top-2 gap is within 2e-2 (each such
exemption is printed).
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from engine import Qwen3VLDecodeEngine, hf_inv_freq
from oracle.qwen3vl_oracle import Qwen3VLOracle
from qwen3vl_config import QWEN3VL_2B, synthetic_prompt, synthetic_state, vision_grid_positions

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
LOGIT_ATOL = 2e-2
LOGIT_MEAN_28L = 5e-3


def _teacher_forced_check(eng, oracle, prompt, n_new, pos3=None, rope_delta=0, atol=LOGIT_ATOL, mean_tol=None,
                          tie_tol=LOGIT_ATOL):
    """Greedy-decode `n_new` tokens on the GPU, run the oracle teacher-forced
    on the GPU's tokens, and check every step.  Returns (tokens, logits, per-step
    max |d|, per-step mean |d|, steps whose token differs from the oracle's
    argmax only inside a near-tie, oracle logits)."""
    toks = eng.generate(prompt, n_new, pos3=pos3).numpy()
    P = len(prompt)
    gl = np.stack([eng.step_logits(P - 1 + i).float().cpu().numpy() for i in range(n_new)])
    otoks, ol = oracle.greedy(prompt, n_new, pos3_prompt=pos3, rope_delta=rope_delta, forced=toks)
    d = np.abs(gl - ol)
    diff, mean = d.max(axis=-1), d.mean(axis=-1)
    q = np.quantile(diff, [0.5, 0.9, 0.99])
    print(f"\n{n_new} steps: max |d logit| {diff.max():.4g} (step {int(diff.argmax())}), median {q[0]:.4g}, "
          f"p90 {q[1]:.4g}, p99 {q[2]:.4g}; mean |d| max {mean.max():.4g}; steps above {LOGIT_ATOL}: "
          f"{int((diff > LOGIT_ATOL).sum())}; token differences from the oracle's argmax: {int((toks != otoks).sum())}")
    assert diff.max() <= atol, f"max logit diff per step {diff}"
    if mean_tol is not None:
        assert mean.max() <= mean_tol, f"mean logit diff per step {mean}"
    srt = np.sort(ol, axis=-1)
    gap = srt[:, -1] - srt[:, -2]
    exempt = []
    for i in range(n_new):
        if toks[i] != otoks[i]:
            assert gap[i] <= tie_tol, f"step {i}: token {toks[i]} vs oracle {otoks[i]} (gap {gap[i]})"
            exempt.append((i, int(toks[i]), int(otoks[i]), float(gap[i])))
    # the engine's token is the first max of its own fp16 logits
    np.testing.assert_array_equal(toks, np.argmax(gl, axis=-1))
    return toks, gl, diff, mean, exempt, ol


@pytest.fixture(scope="module")
def state2():
    return synthetic_state(QWEN3VL_2B.with_layers(2), seed=0)


def test_engine_matches_reference_golden_text(cuda_device, state2):
    g = np.load(GOLDEN / "greedy_text.npz")
    n = len(g["tokens"])
    eng = Qwen3VLDecodeEngine(state2, QWEN3VL_2B.with_layers(2), max_cache_len=128, logits_ring=n,
                              max_steps=128)
    toks = eng.generate(g["prompt"], n).numpy()
    np.testing.assert_array_equal(toks, g["tokens"])
    P = len(g["prompt"])
    gl = np.stack([eng.step_logits(P - 1 + i).float().cpu().numpy() for i in range(n)])
    assert np.abs(gl[:, g["sample_idx"]] - g["sample_logits"]).max() <= 5e-2


def test_engine_matches_reference_golden_vision_grid(cuda_device, state2):
    g = np.load(GOLDEN / "vision_grid.npz")
    n = len(g["tokens"])
    eng = Qwen3VLDecodeEngine(state2, QWEN3VL_2B.with_layers(2), max_cache_len=320, logits_ring=n,
                              max_steps=512)
    toks = eng.generate(g["prompt"], n, pos3=g["pos3"]).numpy()
    np.testing.assert_array_equal(toks, g["tokens"])


def test_engine_two_layers_teacher_forced(cuda_device, state2):
    s16 = {k: v.half() for k, v in state2.items()}
    prompt = synthetic_prompt(200, seed=77).numpy()
    eng = Qwen3VLDecodeEngine(s16, QWEN3VL_2B.with_layers(2), max_cache_len=512, logits_ring=64, max_steps=512)
    o = Qwen3VLOracle(s16, 2, mode="fp16", max_cache_len=512, inv_freq=hf_inv_freq(QWEN3VL_2B).numpy())
    _teacher_forced_check(eng, o, prompt, 64)


def test_engine_cuda_graph_replay_is_deterministic(cuda_device, state2):
    prompt = synthetic_prompt(40, seed=5).numpy()
    eng = Qwen3VLDecodeEngine(state2, QWEN3VL_2B.with_layers(2), max_cache_len=256, max_steps=256)
    a = eng.generate(prompt, 70, graph_steps=16)
    b = eng.generate(prompt, 70, graph_steps=1)
    c = eng.generate(prompt, 70, graph_steps=32)
    assert torch.equal(a, b) and torch.equal(a, c)


def test_engine_device_side_eos(cuda_device, state2):
    """A generated token equal to eos_token_id ends the request on the
    device: generate() returns the tokens up to and including it, the step
    state stops advancing (later launches, graph replays included, return at
    once) and a request without EOS is unaffected."""
    prompt = synthetic_prompt(40, seed=5).numpy()
    eng = Qwen3VLDecodeEngine(state2, QWEN3VL_2B.with_layers(2), max_cache_len=256, max_steps=256)
    ref = eng.generate(prompt, 40, graph_steps=16)
    assert eng.done_step() == 0
    # EOS = the first generated token not seen before, from the 4th on if any
    k = next((i for i in range(3, len(ref)) if int(ref[i]) not in ref[:i].tolist()), 0)
    eos = int(ref[k])
    got = eng.generate(prompt, 40, graph_steps=16, eos_token_id=eos)
    assert torch.equal(got, ref[:k + 1]), (got, ref[:k + 1])
    P = len(prompt)
    assert eng.done_step() == P + k  # the EOS came out of step P - 1 + k
    st = eng.state_dev.view(torch.int64)
    assert int(st[1]) == P + k  # cache slot of the step after EOS: no later launch advanced it
    again = eng.generate(prompt, 40, graph_steps=16)  # a new request without EOS runs in full
    assert torch.equal(again, ref)


def test_engine_gemm_prefill_then_device_decode(cuda_device, state2):
    """prefill="gemm" (the whole vision-grid prompt in one pass, K/V written
    to the engine's cache) followed by device decode: teacher-forced logits of
    every step against the oracle, and the same tokens as the one-token-per-
    launch prefill up to the first step where the oracle's own top-2 gap is
    within tolerance (a near tie may send the two trajectories apart)."""
    P, n = 300, 12
    pos3, rope_delta = vision_grid_positions(P)
    prompt = synthetic_prompt(P, seed=4321).numpy()
    eng = Qwen3VLDecodeEngine(state2, QWEN3VL_2B.with_layers(2), max_cache_len=P + n, logits_ring=n, max_steps=P + n)
    toks = eng.generate(prompt, n, pos3=pos3.numpy(), prefill="gemm").numpy()
    gl = np.stack([eng.step_logits(P - 1 + i).float().cpu().numpy() for i in range(n)])
    o = Qwen3VLOracle(state2, 2, mode="fp16", max_cache_len=P + n, inv_freq=hf_inv_freq(QWEN3VL_2B).numpy())
    _, ol = o.greedy(prompt, n, pos3_prompt=pos3.numpy(), rope_delta=rope_delta, forced=toks)
    diff = np.abs(gl - ol).max(axis=-1)
    assert diff.max() <= LOGIT_ATOL, f"max logit diff per step {diff}"
    assert np.array_equal(toks, np.argmax(gl, axis=-1))
    ref = eng.generate(prompt, n, pos3=pos3.numpy(), prefill="decode").numpy()
    top2 = np.sort(ol, axis=-1)[:, -2:]
    for i in range(n):
        if toks[i] != ref[i]:
            assert top2[i, 1] - top2[i, 0] <= 2 * LOGIT_ATOL, (i, toks[i], ref[i])
            break


def test_engine_full_model_benchmarked_request(cuda_device):
    """BASELINE config 4 as bench.py runs it: 28 layers, the bench's 1024-token
    prefix (16x16 vision grid, 3-axis MRoPE), then the first token and the 256
    benchmarked decode steps (257 tokens).

    Checker: the fp16 oracle with float64 sums, teacher-forced on the GPU's
    tokens.  Beside it the same oracle with float32 sums (an independent,
    correct fp32-summing implementation of the same model) gives the noise
    floor of fp32 summation at 28 layers; measured on the CPU over 40 of these
    steps it already reaches max 0.0225 / median 0.0176 per step, so a fixed
    2e-2 per-step max is below what two correct implementations agree to.
    Asserted: every token equal to the oracle's argmax unless the oracle's own
    top-2 gap is within 2e-2 (each such exemption is printed); mean |d logit|
    <= 5e-3 at every step; the median over steps of the per-step max <= 2e-2;
    and the worst step within max(2e-2, 1.15 x the floor's worst step)."""
    import bench

    st = synthetic_state(QWEN3VL_2B, seed=0, dtype=torch.float16)
    prompt, pos3, rope_delta = bench.headline_request(0)
    P, n = bench.PREFIX, bench.NEW + 1
    prompt = prompt.numpy()
    inv = hf_inv_freq(QWEN3VL_2B).numpy()
    eng = Qwen3VLDecodeEngine(st, QWEN3VL_2B, max_cache_len=P + bench.NEW, logits_ring=n, max_steps=P + n)
    o64 = Qwen3VLOracle(st, 28, mode="fp16", max_cache_len=P + n, inv_freq=inv, accumulate="f64")
    toks, gl, diff, mean, exempt, ol64 = _teacher_forced_check(eng, o64, prompt, n, pos3=pos3.numpy(),
                                                               rope_delta=rope_delta, atol=np.inf,
                                                               mean_tol=LOGIT_MEAN_28L)
    del o64, eng
    o32 = Qwen3VLOracle(st, 28, mode="fp16", max_cache_len=P + n, inv_freq=inv)
    del st
    _, ol32 = o32.greedy(prompt, n, pos3_prompt=pos3.numpy(), rope_delta=rope_delta, forced=toks)
    del o32
    floor = np.abs(ol32 - ol64).max(axis=-1)
    print(f"noise floor (fp32-sum oracle vs float64-sum oracle, same tokens): max {floor.max():.4g}, "
          f"median {np.median(floor):.4g}; GPU vs float64-sum oracle: max {diff.max():.4g}, "
          f"median {np.median(diff):.4g}")
    print(f"28-layer benchmarked request: near-tie exemptions {len(exempt)}: {exempt}")
    print("per-step max |d| GPU:", " ".join(f"{x:.4f}" for x in diff))
    print("per-step max |d| floor:", " ".join(f"{x:.4f}" for x in floor))
    assert np.median(diff) <= LOGIT_ATOL, np.median(diff)
    assert diff.max() <= max(LOGIT_ATOL, 1.15 * floor.max()), (diff.max(), floor.max())
