"""GPU parity at the reference's own model configuration (main.py:27-65): seq_len 384,
model_dim 128 with 4 heads (head_dim F = 32), the F x F inner MLP of ttt_layer.py:427-430,
mini_batch_size CS = 64, base learning rate 0.05, checkpoint group 16, memo segments of 2
mini-batches, batch 32, trained under fp16 autocast (main.py:87).

Outside the tensor-core envelope (CS = 16, F = 64), these shapes run on the general
kernels (ttt_mlp.cu) and the segment loop on the cached read-out kernel; every output and
gradient is checked here against the oracle and the reference's own forecaster goldens."""

import math

import pytest
import torch

import synthetic as S
import ttt_oracle as O
from forecaster import TTTForecaster, load_reference_state_dict, make_optimizer, train_step
from helpers import TOL, assert_close, load_golden, oracle_inputs, to_dev
from mlp_triton import TritonMLP

pytestmark = pytest.mark.gpu
DEV = "cuda"
NAMES = ("ln_w", "ln_b", "W1", "b1", "W2", "b2", "XQ", "XV", "XK", "eta")
# main.py: batch 32, 4 heads, 384 / 64 = 6 mini-batches of 64 tokens, head_dim 32, F x F
B, NH, NC, CS, F, FF, CKPT, MEMO = 32, 4, 6, 64, 32, 32, 16, 2


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("eta_mode", ["equal", "causal"])
def test_triton_mlp_forward_and_gradients_at_main_config(dtype, eta_mode):
    """TritonMLP.apply at main.py's shape: XQW, all twelve gradients, the memo states (after
    mini-batches 0, 2, 4) and the final state against the fp64 oracle. `equal` eta is what
    the forecaster's layer feeds (ttt_layer.py:309)."""
    d = S.perturb_params(S.make_mlp_inputs(B, NH, NC, CS, F, FF, seed=90, eta_mode=eta_mode), seed=91)
    d = to_dev(d, DEV, dtype)
    dO = S.make_upstream((B, NH, NC, CS, F), seed=92).to(DEV, dtype)
    leaves = {k: d[k].detach().clone().requires_grad_(True) for k in NAMES}
    out, *memos = TritonMLP.apply(*(leaves[k] for k in NAMES), min(CKPT, NC), MEMO)
    out.backward(dO)
    od = oracle_inputs(d)
    ref_grads, ref = O.mlp_grads(od, dO.double().cpu())
    full = O.mlp_scan(*(od[k] for k in NAMES), min(CKPT, NC), MEMO)
    tol = TOL[dtype]
    assert out.dtype == dtype and out.shape == (B, NH, NC, CS, F)
    assert_close("XQW", out, ref["XQW"], tol)
    for k in NAMES:
        assert leaves[k].grad.dtype == d[k].dtype, k
        assert_close("d" + k, leaves[k].grad, ref_grads[k], tol)
    assert memos[0].shape[2] == math.ceil(NC / MEMO)
    for i, name in enumerate(("W1", "b1", "W2", "b2")):
        assert_close(name + "_memo", memos[i], full[name + "_memo"], tol)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_memo_mixing_at_main_config(dtype):
    """The layer's memo mixing (3 segments of 2 mini-batches of 64 tokens, F x F memo states
    of head_dim 32) through mlp_memo_mix: output and the gradients of XQW, XU, XK."""
    from kernels.mlp_memo_mix import fused_envelope, mlp_memo_mix

    d = S.perturb_params(S.make_mlp_inputs(B, NH, NC, CS, F, FF, seed=93, eta_mode="equal"), seed=94)
    od = {k: v.double() for k, v in d.items()}
    r = O.mlp_scan(*(od[k] for k in NAMES), 1, MEMO)
    g = torch.Generator().manual_seed(95)
    XU = torch.randn(B, NH, NC, CS, F, generator=g)
    inp = {"XQW": r["XQW"].to(dtype), "XQ": d["XQ"].to(dtype), "XK": d["XK"].to(dtype), "XU": XU.to(dtype),
           "W1_memo": r["W1_memo"].float(), "b1_memo": r["b1_memo"].float(), "W2_memo": r["W2_memo"].float(),
           "b2_memo": r["b2_memo"].float(), "ln_w": d["ln_w"], "ln_b": d["ln_b"]}
    order = ("XQW", "XQ", "XK", "XU", "W1_memo", "b1_memo", "W2_memo", "b2_memo", "ln_w", "ln_b")
    dO = S.make_upstream((B, NH, NC, CS, F), seed=96).to(dtype)
    leaves = {k: v.to(DEV).requires_grad_(k in ("XQW", "XU", "XK")) for k, v in inp.items()}
    assert not fused_envelope(leaves["XQW"], leaves["W1_memo"], MEMO)
    out = mlp_memo_mix(*(leaves[k] for k in order), MEMO)
    out.backward(dO.to(DEV))
    ref_g, ref = O.memo_mix_grads({k: v.double() for k, v in inp.items()}, dO.double(), MEMO)
    tol = TOL[dtype]
    assert_close("out", out, ref, tol)
    for k in ("XQW", "XU", "XK"):
        assert_close("d" + k, leaves[k].grad, ref_g[k], tol)


def golden_model(name, act_dtype):
    inp, g = load_golden(name)
    P = {k[2:]: v for k, v in g.items() if k.startswith("p_")}
    L, d_in = inp["x"].shape[1], inp["x"].shape[2]
    W = P["in_proj.weight"].shape[0]
    model = TTTForecaster(d_in, d_in, int(g["pred_len"]), L, model_dim=W, num_heads=int(g["NH"]), num_layers=1,
                          mini_batch_size=int(g["CS"]), ttt_base_lr=float(g["base_lr"]),
                          scan_checkpoint_group_size=int(g["ckpt"]), mem_cache_segment_n_mini_batches=int(g["memo"]),
                          act_dtype=act_dtype)
    load_reference_state_dict(model, P)
    return model.to(DEV), inp, g


@pytest.mark.parametrize("act_dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("name", ["forecaster_main", "forecaster_main_memo"])
def test_forecaster_matches_reference_at_main_config(name, act_dtype):
    """The reference's own TTTForecaster built from main.py's ModelConfig (goldens from
    tests/golden/make_golden.py): output, MSE loss and the gradient of every parameter. The
    `_memo` golden mixes three memo segments through the reference's cached read-out
    kernel (B = NH = 1, the slice it addresses correctly)."""
    model, inp, g = golden_model(name, act_dtype)
    out = model(inp["x"].to(DEV))
    loss = torch.nn.functional.mse_loss(out.float(), inp["y"].to(DEV))
    loss.backward()
    tol = TOL[act_dtype]
    assert_close("out", out, g["out"], tol)
    assert abs(float(loss.detach()) - float(g["loss"])) <= tol * abs(float(g["loss"]))
    for pname, p in model.named_parameters():
        ref_name = "ttt.ttt." + pname[len("layers.0."):] if pname.startswith("layers.0.") else pname
        assert_close("grad " + pname, p.grad, g["g_" + ref_name], tol)


def test_training_steps_of_the_main_py_model():
    """main.py's model (one TTT-MLP layer, d 128, 4 heads, CS 64, lr 0.05) on fp16
    activations: training steps on a fixed batch of 32 windows of 384 lower the loss."""
    torch.manual_seed(0)
    series = S.make_forecast_series(4000, 1, seed=3)
    x, y = S.forecast_windows(series, 384, 96, 32, torch.Generator().manual_seed(4))
    model = TTTForecaster(1, 1, 96, 384, model_dim=128, num_heads=4, num_layers=1, mini_batch_size=64,
                          ttt_base_lr=0.05, scan_checkpoint_group_size=16, mem_cache_segment_n_mini_batches=2,
                          act_dtype=torch.float16).to(DEV)
    opt = make_optimizer(model)
    losses = [float(train_step(model, opt, x.to(DEV), y.to(DEV))) for _ in range(6)]
    assert all(math.isfinite(v) for v in losses)
    assert losses[-1] < losses[0]


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_triton_linear_at_main_config(dtype):
    """TritonLinear.apply (the ModelConfig default ssm_layer, ttt_linear) at main.py's shape:
    XQW and all ten gradients against the oracle."""
    from linear_triton import TritonLinear

    names = ("ln_w", "ln_b", "W1", "b1", "XQ", "XV", "XK", "eta")
    d = S.perturb_params(S.make_linear_inputs(B, NH, NC, CS, F, seed=97, eta_mode="equal"), seed=98)
    d = to_dev(d, DEV, dtype)
    # upstream gradient at the scale of a training loss: N(0, 1) per element with CS = 64 drives
    # d_eta past the fp16 range (65504) in fp64 too
    dO = (S.make_upstream((B, NH, NC, CS, F), seed=99) * 0.01).to(DEV, dtype)
    leaves = {k: d[k].detach().clone().requires_grad_(True) for k in names}
    out = TritonLinear.apply(*(leaves[k] for k in names), min(CKPT, NC))
    out.backward(dO)
    ref_grads, ref = O.linear_grads(oracle_inputs(d), dO.double().cpu())
    tol = TOL[dtype]
    assert_close("XQW", out, ref["XQW"], tol)
    for k in names:
        assert_close("d" + k, leaves[k].grad, ref_grads[k], tol)
