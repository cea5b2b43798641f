"""GPU parity of the memo read-out (mlp_cached_readout_triton drop-in)."""

import pytest
import torch

import synthetic as S
import ttt_oracle as O
from helpers import assert_close, load_golden, oracle_inputs, to_dev
from kernels.mlp_cached_readout import mlp_cached_readout_triton
from mlp_triton import TritonMLP

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_readout_matches_reference_kernel_golden():
    inp, g = load_golden("cached_readout")
    d = to_dev(inp, DEV)
    out = mlp_cached_readout_triton(d["XQ"], d["W1"], d["b1"], d["W2"], d["b2"], d["ln_w"], d["ln_b"])
    assert out.dtype == torch.float32
    assert_close("readout", out, g["out"], 1e-5)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_readout_on_memo_slices_every_head(dtype):
    """Non-contiguous memo slices W*_memo[:, :, j] as the layer passes them; every (b, h)
    gets its own output (the shipped kernel only fills (0, 0))."""
    B, NH, NC, CS, F, FF = 2, 3, 6, 16, 32, 128
    d = S.perturb_params(S.make_mlp_inputs(B, NH, NC, CS, F, FF, dtype=dtype, device=DEV, seed=4), device=DEV, seed=5)
    names = ("ln_w", "ln_b", "W1", "b1", "W2", "b2", "XQ", "XV", "XK", "eta")
    _, *memo = TritonMLP.apply(*(d[k] for k in names), 2, 2)
    XQ_seg = d["XQ"][:, :, 2:4].contiguous()
    for j in range(memo[0].shape[2]):
        W1, b1, W2, b2 = (m[:, :, j] for m in memo)
        assert not W1.is_contiguous()
        out = mlp_cached_readout_triton(XQ_seg, W1, b1, W2, b2, d["ln_w"], d["ln_b"])
        ref = O.mlp_cached_readout(*(t.detach().double().cpu() for t in (XQ_seg, W1, b1, W2, b2, d["ln_w"], d["ln_b"])))
        assert_close(f"readout j={j}", out, ref, 1e-4 if dtype == torch.float32 else 2e-2)
