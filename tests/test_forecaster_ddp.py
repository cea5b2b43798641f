"""CPU, world_size 2 over gloo: the data-parallel training step the forecaster bench runs
(per-rank batch shard, DistributedDataParallel gradient averaging, identical parameters after
the optimiser step) with a small CPU stand-in model, plus the config-4 series windows."""

import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import synthetic as S
from forecaster import train_step


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.manual_seed(0)  # identical initial parameters on every rank
    model = torch.nn.Sequential(torch.nn.Flatten(), torch.nn.Linear(32 * 7, 8 * 7), torch.nn.Unflatten(1, (8, 7)))
    ddp = torch.nn.parallel.DistributedDataParallel(model)
    opt = torch.optim.AdamW(ddp.parameters(), lr=1e-3, weight_decay=1e-2)
    series = S.make_forecast_series(500, 7, seed=3)
    x, y = S.forecast_windows(series, 32, 8, 8, torch.Generator().manual_seed(5))
    shard = slice(rank * 4, rank * 4 + 4)  # the global batch split over ranks
    train_step(ddp, opt, x[shard], y[shard])
    flat = torch.cat([p.detach().reshape(-1) for p in model.parameters()])
    q.put((rank, flat.numpy().copy()))  # by value: the process exits before the parent reads
    dist.barrier()
    dist.destroy_process_group()


def test_ddp_step_keeps_ranks_identical_and_matches_full_batch():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {r: torch.from_numpy(v) for r, v in (q.get(timeout=120) for _ in range(world))}
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert torch.equal(res[0], res[1])
    # one process on the full batch gives the same update (mean of the shard gradients)
    torch.manual_seed(0)
    model = torch.nn.Sequential(torch.nn.Flatten(), torch.nn.Linear(32 * 7, 8 * 7), torch.nn.Unflatten(1, (8, 7)))
    opt = torch.optim.AdamW(model.parameters(), lr=1e-3, weight_decay=1e-2)
    series = S.make_forecast_series(500, 7, seed=3)
    x, y = S.forecast_windows(series, 32, 8, 8, torch.Generator().manual_seed(5))
    train_step(model, opt, x, y)
    flat = torch.cat([p.detach().reshape(-1) for p in model.parameters()])
    assert torch.allclose(flat, res[0], atol=1e-6)


def test_series_has_the_config4_statistics():
    s = S.make_forecast_series(17420, 7, seed=0)
    assert s.shape == (17420, 7)
    assert torch.allclose(s.mean(0), torch.zeros(7), atol=1e-4)
    assert torch.allclose(s.std(0, unbiased=False), torch.ones(7), atol=1e-3)
    x, y = S.forecast_windows(s, 336, 96, 4, torch.Generator().manual_seed(0))
    assert x.shape == (4, 336, 7) and y.shape == (4, 96, 7)


def test_batch_copies_match_tile_forward_and_backward():
    """BatchCopies (the layer's per-sequence inner-state copies) is torch.tile with the
    batch sum of its backward done as a matrix-vector product."""
    from forecaster import BatchCopies

    torch.manual_seed(1)
    p = torch.randn(4, 8, 16, dtype=torch.float64, requires_grad=True)
    g = torch.randn(5, 4, 8, 16, dtype=torch.float64)
    out = BatchCopies.apply(p, 5)
    ref = torch.tile(p.unsqueeze(0), (5, 1, 1, 1))
    assert out.is_contiguous() and torch.equal(out, ref)
    (gp,) = torch.autograd.grad(out, p, g)
    (gr,) = torch.autograd.grad(ref, p, g)
    assert torch.allclose(gp, gr, rtol=1e-12, atol=1e-12)


def test_linear_act_matches_linear():
    """linear_act (the input projection with K padded to 8, the bias carried by the first
    padding column) equals nn.Linear: output, weight and bias gradients."""
    from forecaster import linear_act

    torch.manual_seed(2)
    for k in (7, 5, 8):
        x = torch.randn(3, 11, k, dtype=torch.float64)
        lin = torch.nn.Linear(k, 16).double()
        y, ref = linear_act(x, lin.weight, lin.bias, torch.float64), lin(x)
        g = torch.randn_like(ref)
        got = torch.autograd.grad(y, (lin.weight, lin.bias), g)
        want = torch.autograd.grad(ref, (lin.weight, lin.bias), g)
        assert torch.allclose(y, ref, rtol=1e-12, atol=1e-12)
        for a, b in zip(got, want):
            assert torch.allclose(a, b, rtol=1e-12, atol=1e-12)
