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
                                   (2, 1, 6, 16, 32, 32, 4, 1), (1, 1, 3, 8, 32, 128, 1, 2),
                                   (2, 3, 5, 16, 64, 64, 2, 2)])
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
    XQW, last, ck, _, _ = _core.mlp_forward(*(d[k] for k in NAMES), ckpt, None)
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
    out, last, _, _, _ = _core.mlp_forward(*(d[k] for k in NAMES), 16, None, for_backward=False)
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


@pytest.mark.parametrize("FF", [256, 64])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("eta_mode", ["causal", "equal"])
def test_backward_paths_agree(dtype, eta_mode, FF):
    """The single reverse walk over the stored pre-activations (tensor-core path, 8 warps for
    the 256-wide inner MLP, 2 for the F x F one) and the checkpoint-group recompute (general
    path) both match the oracle on the same inputs."""
    B, NH, NC, CS, F, ckpt = 2, 2, 7, 16, 64, 3
    d, dO = make(B, NH, NC, CS, F, FF, dtype, seed=31, eta_mode=eta_mode)
    ref_grads, _ = O.mlp_grads(oracle_inputs(d), dO.double().cpu())
    _, last, ck, _, zs = _core.mlp_forward(*(d[k] for k in NAMES), ckpt, None)
    args = (d["ln_w"], d["ln_b"], ck, d["XQ"], d["XV"], d["XK"], d["eta"], dO, ckpt)
    walk = _core.mlp_backward(*args, saved=zs, W1_last=last[0], W2_last=last[2])
    regroup = _core.mlp_backward(*args)
    names = ("ln_w", "ln_b", "W1", "b1", "W2", "b2", "XQ", "XV", "XK", "eta")
    for res in (walk, regroup):
        got = dict(zip(names, res))
        got["ln_w"], got["ln_b"] = got["ln_w"].sum(0), got["ln_b"].sum(0)
        for k in names:
            assert_close("d" + k, got[k], ref_grads[k].reshape(got[k].shape), 2e-2)


@pytest.mark.parametrize("FF", [256, 64])
def test_saved_preactivations_match_oracle(FF):
    """The forward's stored Z1, Z2, Z1bar, Z2bar equal the oracle's per-mini-batch values."""
    B, NH, NC, CS, F = 1, 2, 5, 16, 64
    d, _ = make(B, NH, NC, CS, F, FF, torch.bfloat16, seed=41)
    _, _, _, _, zs = _core.mlp_forward(*(d[k] for k in NAMES), 2, None)
    od = oracle_inputs(d)
    st = [od["W1"], od["b1"], od["W2"], od["b2"]]
    gamma, beta = od["ln_w"].reshape(NH, 1, F), od["ln_b"].reshape(NH, 1, F)
    ref = [[], [], [], []]
    for n in range(NC):
        XQ, XK, XV, eta = (od[k][:, :, n] for k in ("XQ", "XK", "XV", "eta"))
        Z1 = XK @ st[0] + st[1]
        X2 = O.gelu_tanh(Z1)
        Z2 = X2 @ st[2] + st[3]
        G2 = O.ln_fused_l2_bwd(Z2, XV - XK, gamma, beta)
        G1 = (G2 @ st[2].transpose(-1, -2)) * O.gelu_bwd(Z1)
        P1 = eta * (XQ @ XK.transpose(-1, -2) + 1)
        Z1b = XQ @ st[0] + st[1] - P1 @ G1
        X2b = O.gelu_tanh(Z1b)
        P2 = eta * (X2b @ X2.transpose(-1, -2) + 1)
        Z2b = X2b @ st[2] + st[3] - P2 @ G2
        for i, z in enumerate((Z1, Z2, Z1b, Z2b)):
            ref[i].append(z)
        e = eta[:, :, -1, :, None]
        st = [st[0] - (e * XK).transpose(-1, -2) @ G1, st[1] - (e * G1).sum(-2, keepdim=True),
              st[2] - (e * X2).transpose(-1, -2) @ G2, st[3] - (e * G2).sum(-2, keepdim=True)]
    for i, name in enumerate(("Z1", "Z2", "Z1bar", "Z2bar")):
        assert_close(name, zs[i], torch.stack(ref[i], 2), 2e-2)


@pytest.mark.parametrize("FF", [256, 64])
@pytest.mark.parametrize("B,NH", [(1, 2), (2, 150), (4, 64), (8, 160)])
def test_forward_sampled_streams_few_and_many(B, NH, FF):
    """Grids below and above the number of SMs (one and several waves; with FF = 64 several
    2-warp CTAs share an SM's tensor memory): final states, checkpoints, memo states and
    outputs of sampled streams match the oracle."""
    NC, CS, F = 3, 16, 64
    d, _ = make(B, NH, NC, CS, F, FF, torch.bfloat16, seed=B + NH)
    out, last, ck, memo, zs = _core.mlp_forward(*(d[k] for k in NAMES), 2, 1)
    od = oracle_inputs(d)
    for b, hh in ((0, 0), (B - 1, NH - 1), (B // 2, NH // 2)):
        sub = {k: (v[b:b + 1, hh:hh + 1] if k not in ("ln_w", "ln_b") else v[hh:hh + 1]) for k, v in od.items()}
        r = O.mlp_scan(*(sub[k] for k in NAMES), 2, 1)
        assert_close(f"XQW[{b},{hh}]", out[b:b + 1, hh:hh + 1], r["XQW"], 2e-2)
        for i, name in enumerate(("W1", "b1", "W2", "b2")):
            init = sub[name]
            assert_close(f"{name}_last[{b},{hh}]", last[i][b:b + 1, hh:hh + 1].double().cpu() - init,
                         r[name + "_last"] - init, 2e-2)
            assert_close(f"{name}_ckpt[{b},{hh}]", ck[i][b:b + 1, hh:hh + 1], r[name + "_ckpt"], 2e-2)
            assert_close(f"{name}_memo[{b},{hh}]", memo[i][b:b + 1, hh:hh + 1], r[name + "_memo"], 2e-2)


def test_a_wait_that_runs_out_is_reported_and_the_device_stays_usable():
    """With the first stage's copies held back (ttt_test_hold_first_stage) the forward's
    wait for them runs out after 1 ms: the launch completes, the device error word reports
    bit 0, and the next normal launch gives the oracle's results with the word clear."""
    import _lib

    _lib.device_status()
    d, _ = make(2, 3, 4, 16, 64, 256, torch.bfloat16, seed=52)
    _lib.hold_first_stage(True, 1_000_000)
    try:
        _core.mlp_forward(*(d[k] for k in NAMES), 2, None, for_backward=False)
        torch.cuda.synchronize()
    finally:
        _lib.hold_first_stage(False)
    assert _lib.device_status() & 1
    out, _, _, _, _ = _core.mlp_forward(*(d[k] for k in NAMES), 2, None, for_backward=False)
    r = O.mlp_scan(*(oracle_inputs(d)[k] for k in NAMES))
    assert_close("XQW", out, r["XQW"], 2e-2)
    assert _lib.device_status() == 0
    with pytest.raises(RuntimeError, match="wait limit"):
        _lib.hold_first_stage(True, 3_000_000_000)


def test_no_bounded_wait_gave_up():
    """The TMA-staged kernels report a stage that never landed in the device error word;
    after a run it must be clear."""
    import _lib

    _lib.device_status()
    d, _ = make(2, 3, 5, 16, 64, 256, torch.bfloat16, seed=51)
    _core.mlp_forward(*(d[k] for k in NAMES), 2, None, for_backward=False)
    assert _lib.device_status() == 0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_ops_ttt_mlp_gradients_match_oracle(dtype):
    """ops.ttt_mlp (signature and [B, NC, CS, NH, F] output of ops/ttt_mlp.py:70-99) is
    differentiable in every tensor argument: its gradients match the oracle's and come back
    in each argument's own dtype (fp32 parameters get fp32 gradients, as TritonMLP's do)."""
    import ops

    d, dO = make(2, 2, 5, 16, 64, 256, dtype, seed=61)
    leaves = {k: d[k].detach().clone().requires_grad_(True) for k in NAMES}
    out = ops.ttt_mlp(leaves["XK"], leaves["XQ"], leaves["XV"], leaves["eta"], leaves["ln_w"], leaves["ln_b"],
                      leaves["W1"], leaves["b1"], leaves["W2"], leaves["b2"], 2)
    assert out.shape == (2, 5, 16, 2, 64) and out.dtype == dtype
    out.backward(dO.permute(0, 2, 3, 1, 4))
    ref_grads, ref = O.mlp_grads(oracle_inputs(d), dO.double().cpu())
    tol = TOL[dtype]
    assert_close("XQW", out.permute(0, 3, 1, 2, 4), ref["XQW"], tol)
    for k in NAMES:
        assert leaves[k].grad.dtype == d[k].dtype, k
        assert_close("d" + k, leaves[k].grad, ref_grads[k], tol)


def _forward_all(d, ckpt, memo):
    import _lib

    n0 = _lib.launch_count()
    res = _core.mlp_forward(*(d[k] for k in NAMES), ckpt, memo)
    torch.cuda.synchronize()
    return res, _lib.launch_count() - n0


@pytest.mark.parametrize("extra,NC,dtype", [(2, 13, torch.bfloat16), ("third", 9, torch.float16),
                                            (44, 128, torch.bfloat16)])
def test_balanced_schedule_is_bit_identical(extra, NC, dtype):
    """Between M and 4M/3 streams (M = SM count) the FF = 256 forward runs its balanced
    two-launch schedule (two-stream CTAs, pairing swapped between the launches, the state
    handed over in fp32 through W*_last / b*_last). Every output -- XQW, final states,
    checkpoints and memo states split mid-group, stored pre-activations -- equals the
    one-CTA-per-stream launch bit for bit, and sampled streams match the oracle."""
    import _lib

    M = torch.cuda.get_device_properties(0).multi_processor_count
    S_ = M + (M // 3 if extra == "third" else extra)
    B, NH = (2, S_ // 2) if S_ % 2 == 0 else (1, S_)
    CS, F, FF, ckpt, memo = 16, 64, 256, 4, 3
    d, _ = make(B, NH, NC, CS, F, FF, dtype, seed=S_ + NC)
    try:
        _lib.set_forward_schedule(False)
        plain, n_plain = _forward_all(d, ckpt, memo)
    finally:
        _lib.set_forward_schedule(True)
    bal, n_bal = _forward_all(d, ckpt, memo)
    assert (n_plain, n_bal) == (1, 2)
    out_p, *groups_p = plain
    out_b, *groups_b = bal
    assert torch.equal(out_p, out_b)
    for gp, gb in zip(groups_p, groups_b):
        for i, (a, b) in enumerate(zip(gp, gb)):
            assert torch.equal(a, b), i
    od = oracle_inputs(d)
    for b, hh in ((0, 0), (B - 1, NH - 1)):
        sub = {k: (v[b:b + 1, hh:hh + 1] if k not in ("ln_w", "ln_b") else v[hh:hh + 1]) for k, v in od.items()}
        r = O.mlp_scan(*(sub[k] for k in NAMES), ckpt, memo)
        assert_close(f"XQW[{b},{hh}]", out_b[b:b + 1, hh:hh + 1], r["XQW"], 2e-2)
        init = sub["W1"]
        assert_close(f"W1_last[{b},{hh}]", bal[1][0][b:b + 1, hh:hh + 1].double().cpu() - init,
                     r["W1_last"] - init, 2e-2)


def test_forward_schedule_switch_rejects_bad_ratio():
    import _lib

    with pytest.raises(RuntimeError, match="ratio"):
        _lib.set_forward_schedule(True, 500)
    _lib.set_forward_schedule(True, 0)
