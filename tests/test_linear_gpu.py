"""GPU parity of TTT-Linear (forward, backward, final state, checkpoints) against the CPU oracle.

Bars (north star): relative L2 <= 1e-4 with fp32 activations, <= 2e-2 with bf16/fp16
activations (the oracle runs in float64 on the same, already rounded, inputs).
"""

import pytest
import torch

import _core
import synthetic as S
import ttt_oracle as O
from helpers import TOL, assert_close, load_golden, oracle_inputs, to_dev
from linear_triton import TritonLinear

pytestmark = pytest.mark.gpu
DEV = "cuda"
NAMES = ("ln_w", "ln_b", "W1", "b1", "XQ", "XV", "XK", "eta")


def run_autograd(d, ckpt, dO):
    leaves = {k: d[k].detach().clone().requires_grad_(True) for k in NAMES}
    out = TritonLinear.apply(*(leaves[k] for k in NAMES), ckpt)
    out.backward(dO)
    return out.detach(), {k: leaves[k].grad for k in NAMES}


def make(B, NH, NC, CS, F, dtype, seed=0, eta_mode="causal"):
    d = S.perturb_params(S.make_linear_inputs(B, NH, NC, CS, F, seed=seed, eta_mode=eta_mode), seed=seed + 3)
    d = to_dev(d, DEV, dtype)
    dO = S.make_upstream((B, NH, NC, CS, F), seed=seed + 1).to(DEV, dtype)
    return d, dO


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(2, 2, 5, 16, 32, 2), (1, 3, 4, 16, 64, 16), (2, 1, 7, 16, 16, 3), (1, 2, 3, 8, 64, 1)])
def test_linear_fwd_bwd_matches_oracle(dtype, shape):
    B, NH, NC, CS, F, ckpt = shape
    d, dO = make(B, NH, NC, CS, F, dtype, seed=NC)
    out, grads = run_autograd(d, ckpt, dO)
    ref_grads, ref = O.linear_grads(oracle_inputs(d), dO.double().cpu())
    tol = TOL[dtype]
    assert out.dtype == dtype
    assert_close("XQW", out, ref["XQW"], tol)
    for k in NAMES:
        assert grads[k].dtype == d[k].dtype
        assert_close("d" + k, grads[k], ref_grads[k], tol)
    XQW, W_last, b_last, W_ck, b_ck, Zs = _core.linear_forward(*(d[k] for k in NAMES), ckpt)
    full = O.linear_scan(*(oracle_inputs(d)[k] for k in NAMES), ckpt)
    W0 = d["W1"].double().cpu()
    assert_close("W_last - W0", W_last.double().cpu() - W0, full["W_last"] - W0, tol)
    assert_close("b_last", b_last, full["b_last"], tol)
    assert W_ck.shape[2] == -(-NC // ckpt)
    assert_close("W_ckpt", W_ck, full["W_ckpt"], tol)
    assert_close("b_ckpt", b_ck, full["b_ckpt"], tol)


@pytest.mark.parametrize("name", ["linear_small", "linear_equal_eta", "linear_config0_fwd"])
def test_linear_matches_reference_golden(name):
    inp, g = load_golden(name)
    d = to_dev(inp, DEV)
    ckpt = int(g["ckpt"])
    if "dO" in g:
        dO = g["dO"].to(DEV).permute(0, 3, 1, 2, 4).contiguous()  # ops layout -> kernel layout
        out, grads = run_autograd(d, ckpt, dO)
        for k in NAMES:
            assert_close("d" + k, grads[k], g["grad_" + k], 1e-4)
    else:
        out = TritonLinear.apply(*(d[k] for k in NAMES), ckpt)
    assert_close("XQW", out.permute(0, 2, 3, 1, 4), g["out"], 1e-4)


def test_ops_signature_and_layout():
    import ops

    d, dO = make(2, 2, 4, 16, 32, torch.float32, seed=7)
    out = ops.ttt_linear(d["XK"], d["XQ"], d["XV"], d["eta"], d["ln_w"], d["ln_b"], d["W1"], d["b1"], 2)
    assert out.shape == (2, 4, 16, 2, 32)
    ref = O.ttt_linear(*(oracle_inputs(d)[k] for k in ("XK", "XQ", "XV", "eta", "ln_w", "ln_b", "W1", "b1")), 2)
    assert_close("ops.ttt_linear", out, ref, 1e-4)
    out0 = ops.ttt_linear(d["XK"], d["XQ"], d["XV"], d["eta"], d["ln_w"], d["ln_b"], d["W1"], d["b1"], 0)
    assert_close("ckpt=0", out0, ref, 1e-4)


def test_zero_eta_identity():
    d, _ = make(2, 2, 3, 16, 64, torch.float32, seed=9)
    d["eta"] = torch.zeros_like(d["eta"])
    XQW, W_last, b_last, _, _, _ = _core.linear_forward(*(d[k] for k in NAMES), 2, for_backward=False)
    assert torch.equal(W_last, d["W1"]) and torch.equal(b_last, d["b1"])
    lw, lb = d["ln_w"].reshape(1, 2, 1, 1, 64), d["ln_b"].reshape(1, 2, 1, 1, 64)
    ref = d["XQ"] + O.ln_fwd(d["XQ"] @ d["W1"][:, :, None] + d["b1"][:, :, None], lw, lb)
    assert_close("eta=0", XQW, ref, 1e-5)


def test_mixed_dtypes_and_noncontiguous_inputs():
    d, dO = make(2, 2, 4, 16, 32, torch.bfloat16, seed=11)
    d["XV"] = d["XV"].float()  # the layer's LN target promotes XV to fp32 under autocast
    d["eta"] = d["eta"].float()
    d["XQ"] = d["XQ"].transpose(0, 1).contiguous().transpose(0, 1)  # non-contiguous view
    assert not d["XQ"].is_contiguous()
    out, grads = run_autograd(d, 2, dO)
    ref_grads, ref = O.linear_grads(oracle_inputs(d), dO.double().cpu())
    assert_close("XQW", out, ref["XQW"], 2e-2)
    for k in NAMES:
        assert_close("d" + k, grads[k], ref_grads[k], 2e-2)


def test_checkpoint_group_larger_than_sequence():
    d, dO = make(1, 2, 3, 16, 32, torch.float32, seed=13)
    out, grads = run_autograd(d, 8, dO)
    ref_grads, ref = O.linear_grads(oracle_inputs(d), dO.double().cpu())
    assert_close("XQW", out, ref["XQW"], 1e-4)
    assert_close("dXK", grads["XK"], ref_grads["XK"], 1e-4)


def test_full_size_config2_sampled_streams():
    """Config 2 shape (B32 NH8 L4096 F64, bf16) forward+backward on the GPU; three
    (b, h) streams are re-run through the oracle at full length and compared."""
    B, NH, NC, CS, F = 32, 8, 256, 16, 64
    d = S.make_linear_inputs(B, NH, NC, CS, F, dtype=torch.bfloat16, device=DEV, seed=0)
    dO = S.make_upstream((B, NH, NC, CS, F), device=DEV, seed=1, dtype=torch.bfloat16)
    out, grads = run_autograd(d, 16, dO)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    for b, h in ((0, 0), (17, 3), (31, 7)):
        sub = {k: (v[b:b + 1, h:h + 1] if k not in ("ln_w", "ln_b") else v[h:h + 1]) for k, v in d.items()}
        rg, r = O.linear_grads(oracle_inputs(sub), dO[b:b + 1, h:h + 1].double().cpu())
        assert_close(f"XQW[{b},{h}]", out[b:b + 1, h:h + 1], r["XQW"], 2e-2)
        for k in ("XQ", "XK", "XV", "eta", "W1", "b1"):
            assert_close(f"d{k}[{b},{h}]", grads[k][b:b + 1, h:h + 1], rg[k], 2e-2)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_backward_paths_agree(dtype):
    """The single reverse walk over stored Z (tensor-core path) and the checkpoint-group
    recompute (general path) both match the oracle on the same inputs."""
    B, NH, NC, CS, F, ckpt = 2, 2, 7, 16, 64, 3
    d, dO = make(B, NH, NC, CS, F, dtype, seed=21)
    ref_grads, _ = O.linear_grads(oracle_inputs(d), dO.double().cpu())
    _, Wl, bl, Wc, bc, Z = _core.linear_forward(*(d[k] for k in NAMES), ckpt)
    args = (d["ln_w"], d["ln_b"], Wc, bc, d["XQ"], d["XV"], d["XK"], d["eta"], dO, ckpt)
    walk = _core.linear_backward(*args, Z=Z, W_last=Wl, b_last=bl)
    regroup = _core.linear_backward(*args)
    names = ("ln_w", "ln_b", "W1", "b1", "XQ", "XV", "XK", "eta")
    for res in (walk, regroup):
        got = dict(zip(names, res))
        got["ln_w"], got["ln_b"] = got["ln_w"].sum(0), got["ln_b"].sum(0)
        for k in names:
            assert_close("d" + k, got[k], ref_grads[k].reshape(got[k].shape), 2e-2)


def test_inference_forward_skips_saved_state():
    d, _ = make(1, 2, 3, 16, 64, torch.bfloat16, seed=23)
    with torch.no_grad():
        out = TritonLinear.apply(*(d[k] for k in NAMES), 2)
    XQW, W_last, b_last, W_ck, b_ck, Z = _core.linear_forward(*(d[k] for k in NAMES), 2, for_backward=False)
    assert W_ck is None and b_ck is None and Z is None
    assert torch.equal(out, XQW)
