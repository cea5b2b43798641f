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


def _shard_worker(rank, world, port, q):
    sys.path.insert(0, os.path.join(REPO, "ttt-triton_b200"))
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sharding
        import synthetic as S
        import ttt_oracle as O

        torch.set_num_threads(1)
        names = O.MLP_GRAD_NAMES
        g = {k: v.double() for k, v in S.perturb_params(S.make_mlp_inputs(5, 2, 3, 8, 16, 32, seed=7), seed=8).items()}
        gO = S.make_upstream((5, 2, 3, 8, 16), seed=9).double()
        d = sharding.shard(g, rank, world)
        b0, b1 = sharding.batch_range(5, rank, world)
        grads, out = O.mlp_grads(d, gO[b0:b1].contiguous())
        # per-(b, h) results are gathered; the shared LayerNorm gradients are partial sums
        full_out = sharding.gather(out["XQW"], world)
        full_dxk = sharding.gather(grads["XK"], world)
        dln = grads["ln_w"].clone()
        dist.all_reduce(dln)
        ref_g, ref = O.mlp_grads(g, gO)
        q.put((rank, O.rel_l2(full_out, ref["XQW"]), O.rel_l2(full_dxk, ref_g["XK"]), O.rel_l2(dln, ref_g["ln_w"]),
               b1 - b0))
    finally:
        dist.destroy_process_group()


def test_batch_sharded_streams_equal_unsharded_over_two_gloo_ranks():
    """One global [B, NH, ...] problem (B = 5: ranks hold 2 and 3 batches) split by
    sharding.shard, each rank running the scan on its slice: the gathered outputs and
    per-(b, h) gradients equal the unsharded run, and the all-reduced LayerNorm-weight
    gradient partials equal its batch-summed gradient."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 30500 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_shard_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        assert p.exitcode == 0
    got = sorted(q.get(timeout=5) for _ in range(2))
    assert [g[4] for g in got] == [2, 3]
    for _, e_out, e_dxk, e_ln, _ in got:
        assert e_out < 1e-12 and e_dxk < 1e-12 and e_ln < 1e-12


def test_batch_range_balances_and_covers():
    sys.path.insert(0, os.path.join(REPO, "ttt-triton_b200"))
    import sharding

    for B in (1, 5, 16, 64):
        for world in (1, 2, 4, 8):
            r = [sharding.batch_range(B, k, world) for k in range(world)]
            assert r[0][0] == 0 and r[-1][1] == B
            assert all(r[k][1] == r[k + 1][0] for k in range(world - 1))
            sizes = [b1 - b0 for b0, b1 in r]
            assert max(sizes) - min(sizes) <= 1
