"""Multi-rank host logic of bench.py on CPU: two gloo ranks agree on the
slowest rank's time, the aggregate is whole-job tokens per second, and the
reference arm does its work on rank 0 only."""
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


def _rank(rank, world, port, out):
    import datetime
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        local_ms = [12.5, 20.0][rank]
        out[rank] = bench.reduce_max(local_ms, world, "cpu")
    finally:
        dist.destroy_process_group()


def test_two_rank_max_and_aggregate():
    sys.path.insert(0, ROOT)
    import bench
    port = _free_port()
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    assert out[0] == out[1] == 20.0
    # 2 ranks x 100 steps in the slowest rank's 20 ms -> 10,000 tok/s
    assert bench.aggregate_tok_s(2, 100, out[0] / 1e3) == pytest.approx(10000.0)


def test_reference_arm_runs_on_rank0_only():
    sys.path.insert(0, ROOT)
    import bench

    class A:
        context, steps, warmup = 64, 1, 3

    assert bench.run_reference(A(), 2, 1) == 0  # returns before any work
