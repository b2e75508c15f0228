"""The multi-GPU bench path on CPU: `bench.py --gpus N` runs one sequence
tensor-parallel over N ranks, times every region as the max over ranks and
reports the job's tokens/s (every rank serves the same tokens). Two `gloo`
ranks here check that reduction and the reference arm's rank handling (only
rank 0 runs and prints)."""
import os
import socket
import sys

import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    import bench
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        local_ms = 100.0 + 50.0 * rank  # the slower rank sets the job time
        ms = bench.max_over_ranks_of(local_ms, world, "cpu")
        value = bench.job_tokens_per_s(ms, 128)
        # The reference arm does its work on rank 0 only; the others return at once.
        other = bench.run_reference(None, rank, world) if rank != 0 else None
        q.put((rank, ms, value, other))
    finally:
        dist.destroy_process_group()


def test_two_ranks_max_over_ranks_and_job_throughput():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    got = sorted(q.get(timeout=5) for _ in range(world))
    for rank, ms, value, other in got:
        assert ms == pytest.approx(150.0)  # max over ranks, seen by every rank
        assert value == pytest.approx(128 / 0.150)  # one sequence served by every rank
        assert other is None


def test_single_rank_needs_no_process_group():
    sys.path.insert(0, ROOT)
    import bench
    assert bench.max_over_ranks_of(12.5, 1, "cpu") == 12.5
    assert bench.job_tokens_per_s(1000.0, 128) == pytest.approx(128.0)
