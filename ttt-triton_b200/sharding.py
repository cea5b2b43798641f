"""Batch sharding of the (batch, head) stream grid over ranks, one process per GPU.

Every (b, h) stream of the TTT scan carries its own inner state and never reads another
stream's data, so a global [B, NH, ...] problem splits over ranks with no collective on
the data path: rank r runs the same kernels on batches [r * B // world, (r + 1) * B // world)
of every per-(b, h) tensor (activations, eta, initial states, upstream gradients). The
LayerNorm parameters [NH, F] are read by every rank; their gradients come back as
per-rank partial sums (linear_triton.py:251-252 sums over the batch), which a training
caller adds together with its other outer-parameter gradients in its one all-reduce.

The reference's only sharding notion is head-sharded tensor parallelism through DTensor
``local_map`` (linear_triton.py:267-357, mlp_triton.py:353-463), kept as ``sharded_mode``
on the autograd wrappers; splitting the batch instead keeps every head's LayerNorm
parameters whole on each rank and balances ranks whenever B is a multiple of the world size.
"""

from __future__ import annotations

import torch

# per-head parameters every rank reads whole (not split)
SHARED = ("ln_w", "ln_b", "ttt_norm_weight", "ttt_norm_bias")


def batch_range(B, rank, world):
    """Batches [b0, b1) of rank `rank` out of `world` (balanced; ranks differ by at most one)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} out of range for world size {world}")
    return rank * B // world, (rank + 1) * B // world


def shard(tensors, rank, world, shared=SHARED):
    """Rank `rank`'s slice of a dict of global per-(b, h) tensors (batch on dim 0, made
    contiguous); the names in `shared` are passed through whole."""
    out = {}
    B = None
    for k, v in tensors.items():
        if k in shared or not isinstance(v, torch.Tensor):
            out[k] = v
            continue
        if B is None:
            B = v.shape[0]
        elif v.shape[0] != B:
            raise ValueError(f"{k} has batch {v.shape[0]}, expected {B}")
        b0, b1 = batch_range(B, rank, world)
        out[k] = v[b0:b1].contiguous()
    return out


def gather(t, world, group=None):
    """Concatenate every rank's batch slice of `t` along dim 0 (all-gather; slices may
    differ by one batch). For checking and collecting results, not on the data path."""
    import torch.distributed as dist

    n = torch.tensor([t.shape[0]], device=t.device)
    sizes = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(sizes, n, group=group)
    sizes = [int(s) for s in sizes]
    m = max(sizes)
    pad = t.new_zeros((m, *t.shape[1:]))
    pad[: t.shape[0]] = t
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad.contiguous(), group=group)
    return torch.cat([p[:s] for p, s in zip(parts, sizes)], dim=0)


__all__ = ["SHARED", "batch_range", "shard", "gather"]
