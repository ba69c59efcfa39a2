"""Host logic of bench.py's multi-GPU path, run as two gloo ranks on the CPU.

Under torchrun every rank decodes its own request on its own GPU (request
data parallelism, no data-path collective); the only cross-rank steps are the
start/stop barriers and the max over ranks of the timings.  These tests run
that logic with world_size 2 over gloo on 127.0.0.1, without a GPU.
"""
import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, q):
    import datetime

    import torch.distributed as dist

    import bench

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        dist.barrier()
        # rank r "took" (r + 1) ms on device and 10 (r + 1) ms end to end
        ms, e2e_ms = bench.max_over_ranks([rank + 1.0, 10.0 * (rank + 1)], world)
        # each rank's own row (rank, device, its ms, its setup s) reaches every rank in rank order
        rows = bench.gather_ranks([rank, 4 + rank, rank + 1.0, 0.5], world)
        per = bench.per_rank_report(rows, 3 * bench.NEW)
        q.put((rank, ms, e2e_ms, bench.job_throughput(3, world, ms), per))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_and_job_throughput_world2():
    import bench

    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    got = sorted(q.get(timeout=5) for _ in range(world))
    for rank, ms, e2e_ms, tps, per in got:
        assert ms == 2.0 and e2e_ms == 20.0, (rank, ms, e2e_ms)  # the slowest rank sets the job time
        # whole-job throughput: 3 requests x 256 tokens on each of 2 ranks in 2 ms
        assert tps == pytest.approx(3 * bench.NEW * 2 / 0.002)
        assert [r["rank"] for r in per] == [0, 1] and [r["device"] for r in per] == [4, 5]
        assert per[1]["tok_s"] == pytest.approx(3 * bench.NEW / 0.002)  # rank 1's own rate


def test_single_rank_needs_no_process_group():
    import bench

    assert bench.max_over_ranks([4.0, 5.0], 1) == [4.0, 5.0]
    assert bench.job_throughput(2, 1, 1000.0) == pytest.approx(2 * bench.NEW)


def test_reference_arm_runs_on_rank0_only(capsys):
    import argparse

    import bench

    args = argparse.Namespace(steps=1, warmup=1)
    bench.run_reference(args, rank=1, world=2)  # other ranks exit without work
    assert capsys.readouterr().out == ""


def test_batch_workload_is_seeded_and_in_range():
    """Config 5's per-request contexts: drawn from U[512, 4096] with a
    rank-dependent seed (the same on every run), and both bench arms describe
    the same workload."""
    import bench

    c0 = bench.batch_contexts(8, 0)
    assert c0 == bench.batch_contexts(8, 0)
    assert c0 != bench.batch_contexts(8, 1)  # each rank decodes its own requests
    assert len(c0) == 8 and all(512 <= c <= 4096 for c in c0)
    cfg = bench.batch_workload_config(8, c0, 2)
    assert cfg["contexts"] == c0 and cfg["batch"] == 8 and cfg["parallelism"] == "request-dp2"
    assert "config 5" in cfg["workload"] and cfg["decode_steps_per_request"] == bench.BATCH_NEW
