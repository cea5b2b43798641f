"""CPU: the multi-rank host logic of bench.py with world_size 2 on the gloo backend.

The (b, h) streams shard across ranks with no data-path collective; the only exchange is
the timing reduction (max over ranks) and the whole-job throughput derived from it.
"""

import os
import sys

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)


def _worker(rank, world, port, q):
    sys.path.insert(0, REPO)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench

        ms, e2e = bench.max_over_ranks([1.0 + rank, 5.0 - rank], world, torch.device("cpu"))
        value = bench.weak_scaling_value(world, 1000, ms)
        q.put((rank, ms, e2e, value))
    finally:
        dist.destroy_process_group()


def test_timing_is_max_over_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    got = sorted(q.get(timeout=5) for _ in range(2))
    for rank, ms, e2e, value in got:
        assert ms == 2.0 and e2e == 5.0
        assert abs(value - 2 * 1000 / 2.0e-3) < 1e-6


def test_single_rank_is_identity():
    sys.path.insert(0, REPO)
    import bench

    assert bench.max_over_ranks([3.0, 4.0], 1, None) == [3.0, 4.0]
    assert bench.weak_scaling_value(1, 500, 1.0) == 500 / 1e-3
