"""GPU parity of the fused input prologue (TTTBase.process_input, ttt_layer.py:261-330)
against the oracle restatement and the reference's own outputs (golden vectors)."""

import pytest
import torch

import synthetic as S
import ttt_oracle as O
from helpers import TOL, assert_close, load_golden
from prologue import process_input, ttt_prologue

pytestmark = pytest.mark.gpu
DEV = "cuda"
OUTS = ("XQ", "XK", "XV", "XU", "eta")
ARGS = O.PROLOGUE_PARAM_NAMES


def run_kernel(inp, douts, CS, base_lr, dtype, which=OUTS):
    """Forward and backward through ttt_prologue; weights and hidden states in `dtype`,
    LayerNorm parameters fp32 (as a layer kept in fp32 under a 16-bit activation dtype)."""
    leaves = {}
    for k in ARGS:
        v = inp[k].to(DEV)
        v = v if k in ("ln_w", "ln_b") else v.to(dtype)
        leaves[k] = v.detach().requires_grad_(True)
    cos, sin = inp["freqs_cos"].to(DEV), inp["freqs_sin"].to(DEV)
    out = ttt_prologue(*(leaves[k] for k in ARGS), (cos, sin), CS, base_lr)
    loss = sum((out[k].float() * douts[k].to(DEV, dtype).float()).sum() for k in which)
    loss.backward()
    return out, {k: leaves[k].grad for k in ARGS}


def oracle(inp, douts, CS, base_lr, dtype, which=OUTS):
    """fp64 oracle on the inputs the kernel saw (16-bit rounding applied to hidden and weights)."""
    od = {k: (v if k in ("ln_w", "ln_b", "freqs_cos", "freqs_sin") else v.to(dtype)).double() for k, v in inp.items()}
    dd = {k: (douts[k].to(dtype).double() if k in which else torch.zeros_like(douts[k], dtype=torch.float64))
          for k in OUTS}
    return O.process_input_grads(od, dd, CS, base_lr)


def check(inp, CS, base_lr, dtype, seed, which=OUTS):
    B, L, W = inp["hidden"].shape
    NH = inp["ln_w"].shape[0]
    F = W // NH
    NC = L // CS
    shapes = {"XQ": (B, NH, NC, CS, F), "XK": (B, NH, NC, CS, F), "XV": (B, NH, NC, CS, F),
              "XU": (B, NH, NC, CS, F), "eta": (B, NH, NC, CS, CS)}
    douts = {k: S.make_upstream(shapes[k], seed=seed + i) for i, k in enumerate(OUTS)}
    out, grads = run_kernel(inp, douts, CS, base_lr, dtype, which)
    rg, rout = oracle(inp, douts, CS, base_lr, dtype, which)
    tol = TOL[dtype]
    for k in OUTS:
        assert out[k].dtype == dtype and tuple(out[k].shape) == shapes[k]
        assert_close(k, out[k], rout[k], tol)
    for k in ARGS:
        assert_close("grad " + k, grads[k], rg[k], tol)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(2, 64, 256, 4, 16), (1, 48, 128, 4, 16), (1, 32, 256, 2, 16), (3, 16, 64, 4, 8)])
def test_prologue_matches_oracle(dtype, shape):
    """Outputs and every parameter gradient, head_dim 64 / 32 / 128 / 16, one to several
    mini-batches, mini-batch 16 and 8."""
    B, L, W, NH, CS = shape
    inp = S.make_prologue_inputs(B, L, W, NH, seed=L + W)
    check(inp, CS, 0.1, dtype, seed=5)


def test_prologue_matches_reference_golden():
    """fp32 kernel on the reference's own inputs (its 3-D rotary table included) against the
    outputs and gradients its process_input produced."""
    inp, g = load_golden("prologue")
    CS, base_lr = int(g["CS"]), float(g["base_lr"])
    douts = {k: g["d_" + k] for k in OUTS}
    out, grads = run_kernel(inp, douts, CS, base_lr, torch.float32)
    for k in OUTS:
        assert_close(k, out[k], g["out_" + k], TOL[torch.float32])
    for k in ARGS:
        assert_close("grad " + k, grads[k], g["grad_" + k], TOL[torch.float32])


def test_unused_outputs_and_zero_rows():
    """Only XQ, XK, XV feed the loss (TTT-Linear ignores XU, and eta gets no gradient here):
    the missing gradients reach the kernel as NULL. One token's hidden row and the q bias
    are zero, so its q projection sits on the L2-normalisation clamp."""
    inp = S.make_prologue_inputs(1, 32, 256, 4, seed=9)
    inp["hidden"][0, 5] = 0
    inp["bq"].zero_()
    check(inp, 16, 0.1, torch.float32, seed=11, which=("XQ", "XK", "XV"))


def test_process_input_drop_in_matches_function():
    """process_input(layer, ...) reads a reference-shaped layer's attributes."""

    class Lin:
        def __init__(self, w, b):
            self.weight, self.bias = w, b

    inp = {k: v.to(DEV) for k, v in S.make_prologue_inputs(2, 32, 128, 2, seed=3).items()}
    layer = type("Layer", (), {})()
    for k in ("q", "k", "v", "u"):
        setattr(layer, "w" + k, Lin(inp["w" + k], inp["b" + k]))
    layer.learnable_ttt_lr_weight, layer.learnable_ttt_lr_bias = inp["lr_w"], inp["lr_b"]
    layer.ttt_norm_weight, layer.ttt_norm_bias = inp["ln_w"], inp["ln_b"]
    layer.mini_batch_size, layer.ttt_base_lr, layer.tp_mesh = 16, 0.1, None
    freqs = torch.polar(torch.ones_like(inp["freqs_cos"]), torch.atan2(inp["freqs_sin"], inp["freqs_cos"]))
    got = process_input(layer, inp["hidden"], freqs, None)
    want = ttt_prologue(*(inp[k] for k in ARGS), (inp["freqs_cos"], inp["freqs_sin"]), 16, 0.1)
    for k in OUTS:
        assert torch.allclose(got[k], want[k], rtol=1e-5, atol=1e-6), k
    meta = type("Meta", (), {"is_multiscene": True})()
    with pytest.raises(NotImplementedError):
        process_input(layer, inp["hidden"], freqs, meta)
    with pytest.raises(ValueError):
        ttt_prologue(*(inp[k] for k in ARGS), (inp["freqs_cos"], inp["freqs_sin"]), 24, 0.1)
