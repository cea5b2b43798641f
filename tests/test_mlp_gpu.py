"""GPU parity of TTT-MLP (forward incl. memo/checkpoints, backward) against the CPU oracle."""

import math

import pytest
import torch

import _core
import synthetic as S
import ttt_oracle as O
from helpers import TOL, assert_close, load_golden, oracle_inputs, to_dev
from mlp_triton import TritonMLP

pytestmark = pytest.mark.gpu
DEV = "cuda"
NAMES = ("ln_w", "ln_b", "W1", "b1", "W2", "b2", "XQ", "XV", "XK", "eta")


def make(B, NH, NC, CS, F, FF, dtype, seed=0, eta_mode="causal"):
    d = S.perturb_params(S.make_mlp_inputs(B, NH, NC, CS, F, FF, seed=seed, eta_mode=eta_mode), seed=seed + 3)
    d = to_dev(d, DEV, dtype)
    dO = S.make_upstream((B, NH, NC, CS, F), seed=seed + 1).to(DEV, dtype)
    return d, dO


def run_autograd(d, ckpt, memo, dO):
    leaves = {k: d[k].detach().clone().requires_grad_(True) for k in NAMES}
    out, *memos = TritonMLP.apply(*(leaves[k] for k in NAMES), ckpt, memo)
    out.backward(dO)
    return out.detach(), memos, {k: leaves[k].grad for k in NAMES}


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(2, 2, 5, 16, 16, 64, 2, 2), (1, 2, 4, 16, 64, 256, 16, 3),
                                   (2, 1, 6, 16, 32, 32, 4, 1), (1, 1, 3, 8, 32, 128, 1, 2)])
def test_mlp_fwd_bwd_matches_oracle(dtype, shape):
    B, NH, NC, CS, F, FF, ckpt, memo = shape
    d, dO = make(B, NH, NC, CS, F, FF, dtype, seed=NC + F)
    out, memos, grads = run_autograd(d, ckpt, memo, dO)
    od = oracle_inputs(d)
    ref_grads, ref = O.mlp_grads(od, dO.double().cpu())
    full = O.mlp_scan(*(od[k] for k in NAMES), ckpt, memo)
    tol = TOL[dtype]
    assert_close("XQW", out, ref["XQW"], tol)
    for k in NAMES:
        assert_close("d" + k, grads[k], ref_grads[k], tol)
    NS = math.ceil(NC / memo)
    for i, name in enumerate(("W1", "b1", "W2", "b2")):
        assert memos[i].shape[2] == NS
        assert_close(name + "_memo", memos[i], full[name + "_memo"], tol)
    XQW, last, ck, _ = _core.mlp_forward(*(d[k] for k in NAMES), ckpt, None)
    for i, name in enumerate(("W1", "b1", "W2", "b2")):
        init = od[name]
        assert_close(name + "_last - init", last[i].double().cpu() - init, full[name + "_last"] - init, tol)
        assert_close(name + "_ckpt", ck[i], full[name + "_ckpt"], tol)


@pytest.mark.parametrize("name", ["mlp_small", "mlp_fxf_equal_eta"])
def test_mlp_matches_reference_golden(name):
    inp, g = load_golden(name)
    d = to_dev(inp, DEV)
    dO = g["dO"].to(DEV).permute(0, 3, 1, 2, 4).contiguous()
    out, _, grads = run_autograd(d, int(g["ckpt"]), 1, dO)
    assert_close("XQW", out.permute(0, 2, 3, 1, 4), g["out"], 1e-4)
    for k in NAMES:
        assert_close("d" + k, grads[k], g["grad_" + k], 1e-4)


def test_mlp_triton_back_fxf_and_ops():
    import mlp_triton_back
    import ops

    d, dO = make(2, 2, 4, 16, 32, 32, torch.float32, seed=5)
    leaves = {k: d[k].detach().clone().requires_grad_(True) for k in NAMES}
    out = mlp_triton_back.TritonMLP.apply(*(leaves[k] for k in NAMES), 2)
    out.backward(dO)
    od = oracle_inputs(d)
    ref_grads, ref = O.mlp_grads(od, dO.double().cpu())
    assert_close("XQW", out, ref["XQW"], 1e-4)
    for k in NAMES:
        assert_close("d" + k, leaves[k].grad, ref_grads[k], 1e-4)
    o2 = ops.ttt_mlp(d["XK"], d["XQ"], d["XV"], d["eta"], d["ln_w"], d["ln_b"], d["W1"], d["b1"], d["W2"], d["b2"], 3)
    assert o2.shape == (2, 4, 16, 2, 32)
    assert_close("ops.ttt_mlp", o2, ref["XQW"].permute(0, 2, 3, 1, 4), 1e-4)
    with pytest.raises(ValueError):
        d2, _ = make(1, 1, 2, 16, 16, 64, torch.float32)
        mlp_triton_back.TritonMLP.apply(*(d2[k] for k in NAMES), 1)


def test_full_size_config1_sampled_streams():
    """Config 1 (B16 NH12 L2048 F64 FF256, bf16) forward on the GPU; three streams
    re-run through the oracle at full length."""
    B, NH, NC, CS, F, FF = 16, 12, 128, 16, 64, 256
    d = S.make_mlp_inputs(B, NH, NC, CS, F, FF, dtype=torch.bfloat16, device=DEV, seed=0)
    out, last, _, _ = _core.mlp_forward(*(d[k] for k in NAMES), 16, None, for_backward=False)
    torch.cuda.synchronize()
    for b, h in ((0, 0), (7, 5), (15, 11)):
        sub = {k: (v[b:b + 1, h:h + 1] if k not in ("ln_w", "ln_b") else v[h:h + 1]) for k, v in d.items()}
        r = O.mlp_scan(*(oracle_inputs(sub)[k] for k in NAMES))
        assert_close(f"XQW[{b},{h}]", out[b:b + 1, h:h + 1], r["XQW"], 2e-2)
        W1_0 = sub["W1"].double().cpu()
        assert_close(f"W1_last[{b},{h}]", last[0][b:b + 1, h:h + 1].double().cpu() - W1_0, r["W1_last"] - W1_0, 2e-2)


def test_long_sequence_config3_streams_fwd_bwd():
    """Config 3 length (L8192 -> NC 512, F64 FF256, bf16, memo 16) on two streams,
    forward and backward against the oracle."""
    d, dO = make(1, 2, 512, 16, 64, 256, torch.bfloat16, seed=3)
    out, memos, grads = run_autograd(d, 16, 16, dO)
    ref_grads, ref = O.mlp_grads(oracle_inputs(d), dO.double().cpu())
    assert_close("XQW", out, ref["XQW"], 2e-2)
    for k in NAMES:
        assert_close("d" + k, grads[k], ref_grads[k], 2e-2)
