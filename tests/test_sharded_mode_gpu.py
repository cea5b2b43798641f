"""The head-sharded (DTensor ``local_map``) entry of the autograd wrappers, the reference's
``sharded_mode`` (linear_triton.py:267-357, mlp_triton.py:353-463), on a one-rank device mesh:
inputs and states sharded on the head dimension, LayerNorm parameters on dim 0; outputs and
gradients equal the unsharded call's."""

import os
import socket

import pytest
import torch
import torch.distributed as dist

import synthetic as S
from helpers import to_dev

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture
def mesh():
    from torch.distributed.device_mesh import init_device_mesh

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_free_port()), RANK="0", WORLD_SIZE="1")
    dist.init_process_group("nccl", rank=0, world_size=1, device_id=torch.device(DEV, 0))
    try:
        yield init_device_mesh("cuda", (1,))
    finally:
        dist.destroy_process_group()


def _run(cls, names, d, dO, extra, mesh=None):
    from torch.distributed.tensor import Shard, distribute_tensor

    leaves = {k: d[k].detach().clone().requires_grad_(True) for k in names}
    args = leaves
    if mesh is not None:
        args = {k: distribute_tensor(v, mesh, [Shard(0) if k in ("ln_w", "ln_b") else Shard(1)])
                for k, v in leaves.items()}
    res = cls.apply(*(args[k] for k in names), *extra)
    out = res[0] if isinstance(res, tuple) else res
    if mesh is not None:
        out.backward(distribute_tensor(dO, mesh, [Shard(1)]))
        out = out.full_tensor()
    else:
        out.backward(dO)
    grads = {}
    for k in names:
        g = args[k].grad if mesh is not None else leaves[k].grad
        grads[k] = g.full_tensor() if hasattr(g, "full_tensor") else g
    return out.detach(), grads


@pytest.mark.parametrize("kind", ["linear", "mlp"])
def test_sharded_mode_matches_unsharded_on_one_rank(mesh, kind):
    from linear_triton import TritonLinear
    from mlp_triton import TritonMLP

    if kind == "linear":
        cls, names = TritonLinear, ("ln_w", "ln_b", "W1", "b1", "XQ", "XV", "XK", "eta")
        d = S.perturb_params(S.make_linear_inputs(2, 4, 3, 16, 64, seed=70), seed=71)
        extra = (2,)
    else:
        cls, names = TritonMLP, ("ln_w", "ln_b", "W1", "b1", "W2", "b2", "XQ", "XV", "XK", "eta")
        d = S.perturb_params(S.make_mlp_inputs(2, 4, 3, 16, 64, 256, seed=72), seed=73)
        extra = (2, 2)
    d = to_dev(d, DEV, torch.bfloat16)
    dO = S.make_upstream((2, 4, 3, 16, 64), seed=74).to(DEV, torch.bfloat16)
    ref_out, ref_g = _run(cls, names, d, dO, extra)
    assert cls.sharded_mode is False
    cls.sharded_mode = True
    try:
        out, g = _run(cls, names, d, dO, extra, mesh)
    finally:
        cls.sharded_mode = False
    assert torch.equal(out, ref_out)
    for k in names:
        assert torch.equal(g[k], ref_g[k]), k
