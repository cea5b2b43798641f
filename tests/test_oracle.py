"""CPU: the oracle is pinned to the reference and the hand-derived backward to autograd.

* golden vectors (tests/golden/*.npz, made by tests/golden/make_golden.py from the
  reference's own ops/ package and Triton read-out kernel) vs the oracle restatement;
* the hand-derived dual-form backward (oracle/dual_bwd.py, the algorithm of the CUDA
  backward) vs autograd through the oracle, for several checkpoint group sizes;
* finite differences pin the oracle's autograd gradients;
* known answers: eta = 0 leaves the state unchanged; with all eta rows equal the dual
  form equals the primal (update-then-read-out) form.
"""

import pytest
import torch

import dual_bwd as D
import synthetic as S
import ttt_oracle as O
from helpers import load_golden

GOLD_TOL = 1e-6  # goldens are stored as float32


def _ops_out_to_kernel(out):
    return out.permute(0, 3, 1, 2, 4)  # [B,NC,CS,NH,F] -> [B,NH,NC,CS,F]


@pytest.mark.parametrize("name", ["linear_small", "linear_equal_eta", "linear_config0_fwd"])
def test_linear_oracle_matches_reference_golden(name):
    inp, g = load_golden(name)
    d = {k: v.double() for k, v in inp.items()}
    out = O.ttt_linear(d["XK"], d["XQ"], d["XV"], d["eta"], d["ln_w"], d["ln_b"], d["W1"], d["b1"], int(g["ckpt"]))
    assert O.rel_l2(out, g["out"]) < GOLD_TOL
    if "dO" in g:
        grads, _ = O.linear_grads(d, _ops_out_to_kernel(g["dO"].double()))
        for k, v in grads.items():
            assert O.rel_l2(v, g["grad_" + k]) < GOLD_TOL, k


@pytest.mark.parametrize("name", ["mlp_small", "mlp_fxf_equal_eta"])
def test_mlp_oracle_matches_reference_golden(name):
    inp, g = load_golden(name)
    d = {k: v.double() for k, v in inp.items()}
    out = O.ttt_mlp(d["XK"], d["XQ"], d["XV"], d["eta"], d["ln_w"], d["ln_b"], d["W1"], d["b1"], d["W2"], d["b2"],
                    int(g["ckpt"]))
    assert O.rel_l2(out, g["out"]) < GOLD_TOL
    grads, _ = O.mlp_grads(d, _ops_out_to_kernel(g["dO"].double()))
    for k, v in grads.items():
        assert O.rel_l2(v, g["grad_" + k]) < GOLD_TOL, k


def test_cached_readout_oracle_matches_reference_kernel():
    inp, g = load_golden("cached_readout")
    d = {k: v.double() for k, v in inp.items()}
    out = O.mlp_cached_readout(d["XQ"], d["W1"], d["b1"], d["W2"], d["b2"], d["ln_w"], d["ln_b"])
    assert O.rel_l2(out, g["out"]) < 1e-6


def test_memo_mix_oracle_matches_reference_loop():
    """The memo-state mixing restatement against the reference's own loop (TTTMLP.ttt run
    with its Triton cached read-out under the interpreter), output and gradients."""
    inp, g = load_golden("memo_mix")
    inp = {k: v.double() for k, v in inp.items()}
    grads, out = O.memo_mix_grads(inp, g["dO"].double(), int(g["M"]))
    assert O.rel_l2(out, g["out"].double()) < 1e-6
    for k in O.MEMO_MIX_GRAD_NAMES:
        assert O.rel_l2(grads[k], g["grad_" + k].double()) < 1e-6, k


def test_prologue_oracle_matches_reference_process_input():
    """The input-prologue restatement (projections, L2 norm, rotary embedding, LN target,
    eta) against the reference layer's own process_input, outputs and every gradient."""
    inp, g = load_golden("prologue")
    inp = {k: v.double() for k, v in inp.items()}
    douts = {k[2:]: v.double() for k, v in g.items() if k.startswith("d_")}
    grads, out = O.process_input_grads(inp, douts, int(g["CS"]), float(g["base_lr"]))
    for k, v in out.items():
        assert O.rel_l2(v, g["out_" + k].double()) < 1e-6, k
    for k in O.PROLOGUE_PARAM_NAMES:
        assert O.rel_l2(grads[k], g["grad_" + k].double()) < 1e-6, k


def test_epilogue_oracle_matches_reference_forward_tail():
    """The output-epilogue restatement (permute, post_norm, wo) against the reference layer's
    own forward tail, output and every gradient."""
    inp, g = load_golden("epilogue")
    inp = {k: v.double() for k, v in inp.items()}
    grads, out = O.post_norm_wo_grads(inp, g["dout"].double(), float(g["eps"]))
    assert O.rel_l2(out, g["out"].double()) < 1e-6
    for k in O.EPILOGUE_PARAM_NAMES:
        assert O.rel_l2(grads[k], g["grad_" + k].double()) < 1e-6, k


@pytest.mark.parametrize("name", ["forecaster", "forecaster_main", "forecaster_main_memo"])
def test_forecaster_oracle_matches_reference_model(name):
    """The forecaster composition (in_proj, process_input, scan, memo mixing, post_norm + wo,
    head) against the reference's own TTTForecaster: output, loss and every gradient. The
    `forecaster_main*` goldens are main.py's model configuration (CS 64, head_dim 32, base
    learning rate 0.05, one input channel), the `_memo` one with three memo segments mixed
    through the reference's cached read-out kernel."""
    import ttt_oracle as Or
    from forecaster import rope_table_3d

    inp, g = load_golden(name)
    P = {k[2:]: v.double() for k, v in g.items() if k.startswith("p_")}
    L = inp["x"].shape[1]
    F = P["ttt.ttt.W1"].shape[-1]
    cos, sin = rope_table_3d(F, 1, 1, L)
    grads, out, loss = Or.forecaster_grads(P, inp["x"].double(), inp["y"].double(), ["ttt.ttt."], cos.double(),
                                           sin.double(), int(g["pred_len"]), int(g["CS"]), float(g["base_lr"]),
                                           int(g["ckpt"]), int(g["memo"]))
    assert O.rel_l2(out, g["out"].double()) < 1e-6
    assert abs(float(loss) - float(g["loss"])) < 1e-6 * abs(float(g["loss"]))
    for k, v in grads.items():
        assert O.rel_l2(v, g["g_" + k].double()) < 1e-6, k


def test_rope_table_matches_reference_precompute():
    """rope_table_3d restates utils.precompute_freqs_cis_3d: the golden prologue was made with
    the reference's own table at head_dim 64, 1 x 1 latent, 64 frames."""
    from forecaster import rope_table_3d

    inp, _ = load_golden("prologue")
    cos, sin = rope_table_3d(64, 1, 1, 64)
    assert torch.allclose(cos, inp["freqs_cos"], atol=1e-6) and torch.allclose(sin, inp["freqs_sin"], atol=1e-6)


@pytest.mark.parametrize("eta_mode", ["causal", "equal"])
@pytest.mark.parametrize("ckpt", [1, 3, 16])
def test_linear_hand_backward_matches_autograd(eta_mode, ckpt):
    d = S.perturb_params(S.make_linear_inputs(2, 2, 7, 16, 32, eta_mode=eta_mode), seed=5)
    d = {k: v.double() for k, v in d.items()}
    dO = S.make_upstream((2, 2, 7, 16, 32)).double()
    ref, _ = O.linear_grads(d, dO)
    got = D.linear_backward(d, dO, ckpt)
    for k in ref:
        assert O.rel_l2(got[k], ref[k]) < 1e-12, k


@pytest.mark.parametrize("eta_mode", ["causal", "equal"])
@pytest.mark.parametrize("ckpt", [1, 2, 16])
def test_mlp_hand_backward_matches_autograd(eta_mode, ckpt):
    d = S.perturb_params(S.make_mlp_inputs(2, 2, 5, 16, 16, 64, eta_mode=eta_mode), seed=5)
    d = {k: v.double() for k, v in d.items()}
    dO = S.make_upstream((2, 2, 5, 16, 16)).double()
    ref, _ = O.mlp_grads(d, dO)
    got = D.mlp_backward(d, dO, ckpt)
    for k in ref:
        assert O.rel_l2(got[k], ref[k]) < 1e-12, k


def test_oracle_gradients_match_finite_differences():
    torch.manual_seed(0)
    d = S.perturb_params(S.make_linear_inputs(1, 1, 3, 4, 8), seed=3)
    d = {k: v.double() for k, v in d.items()}
    dO = S.make_upstream((1, 1, 3, 4, 8)).double()
    grads, _ = O.linear_grads(d, dO)

    def loss(dd):
        return (O.linear_scan(dd["ln_w"], dd["ln_b"], dd["W1"], dd["b1"], dd["XQ"], dd["XV"], dd["XK"], dd["eta"])["XQW"] * dO).sum()

    h = 1e-6
    for k in ("XQ", "XK", "XV", "eta", "W1", "ln_w"):
        flat = d[k].reshape(-1)
        for idx in (0, flat.numel() // 2, flat.numel() - 1):
            dp = {kk: vv.clone() for kk, vv in d.items()}
            dm = {kk: vv.clone() for kk, vv in d.items()}
            dp[k].reshape(-1)[idx] += h
            dm[k].reshape(-1)[idx] -= h
            fd = (loss(dp) - loss(dm)) / (2 * h)
            an = grads[k].reshape(-1)[idx]
            assert abs(float(fd - an)) <= 1e-6 * max(1.0, abs(float(an))), (k, idx, float(fd), float(an))


def test_zero_eta_leaves_state_unchanged():
    d = S.perturb_params(S.make_mlp_inputs(1, 2, 4, 16, 16, 32), seed=1)
    d = {k: v.double() for k, v in d.items()}
    d["eta"] = torch.zeros_like(d["eta"])
    res = O.mlp_scan(d["ln_w"], d["ln_b"], d["W1"], d["b1"], d["W2"], d["b2"], d["XQ"], d["XV"], d["XK"], d["eta"])
    for k in ("W1", "b1", "W2", "b2"):
        assert torch.equal(res[k + "_last"], d[k])
    lw = d["ln_w"].reshape(2, 1, 1, 16)
    lb = d["ln_b"].reshape(2, 1, 1, 16)
    Z1 = d["XQ"] @ d["W1"][:, :, None] + d["b1"][:, :, None]
    ref = d["XQ"] + O.ln_fwd(O.gelu_tanh(Z1) @ d["W2"][:, :, None] + d["b2"][:, :, None], lw, lb)
    assert O.rel_l2(res["XQW"], ref) < 1e-13


def test_equal_eta_dual_equals_primal():
    """All eta rows equal (what the forecaster feeds): the dual-form read-out equals the
    primal form that updates W first and then reads out (kernels/linear_forward.py:128-145)."""
    d = S.perturb_params(S.make_linear_inputs(2, 2, 5, 16, 32, eta_mode="equal"), seed=2)
    d = {k: v.double() for k, v in d.items()}
    res = O.linear_scan(d["ln_w"], d["ln_b"], d["W1"], d["b1"], d["XQ"], d["XV"], d["XK"], d["eta"])
    lw, lb = d["ln_w"].reshape(2, 1, 32), d["ln_b"].reshape(2, 1, 32)
    W, b = d["W1"], d["b1"]
    outs = []
    for n in range(5):
        XQ, XK, XV, eta = (d[k][:, :, n] for k in ("XQ", "XK", "XV", "eta"))
        G = O.ln_fused_l2_bwd(XK @ W + b, XV - XK, lw, lb)
        e = eta[:, :, -1, :, None]
        W = W - (e * XK).transpose(-1, -2) @ G
        b = b - (e * G).sum(-2, keepdim=True)
        outs.append(XQ + O.ln_fwd(XQ @ W + b, lw, lb))
    assert O.rel_l2(res["XQW"], torch.stack(outs, 2)) < 1e-12


def test_precision_matched_rounding_rounds_values_and_gradients():
    """ttt_oracle.rounding: the identity for None / float32; for bf16 it rounds the value in
    the forward and the gradient reaching it in the backward, in the working dtype."""
    import ttt_oracle as Or

    x = torch.tensor([1.0 + 2.0 ** -10, -3.0 + 2.0 ** -12], dtype=torch.float64, requires_grad=True)
    assert Or.rounding(None)(x) is x and Or.rounding(torch.float32)(x) is x
    r = Or.rounding(torch.bfloat16)
    y = r(x)
    assert y.dtype == torch.float64 and torch.equal(y.detach(), x.detach().to(torch.bfloat16).double())
    g = torch.tensor([1.0 + 2.0 ** -11, 0.5], dtype=torch.float64)
    y.backward(g)
    assert torch.equal(x.grad, g.to(torch.bfloat16).double())
