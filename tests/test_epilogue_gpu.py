"""GPU parity of the fused output epilogue (permute + post_norm + wo, ttt_layer.py:349-350,
563-564) against the oracle restatement and the reference's own outputs (golden vectors)."""

import pytest
import torch

import ttt_oracle as O
from epilogue import output_epilogue, post_norm_wo
from helpers import TOL, assert_close, load_golden

pytestmark = pytest.mark.gpu
DEV = "cuda"
ARGS = O.EPILOGUE_PARAM_NAMES


def inputs(B, NH, NC, CS, F, seed):
    g = torch.Generator().manual_seed(seed)
    W = NH * F
    return {"XQW": torch.randn(B, NH, NC, CS, F, generator=g) * 0.5 + 0.1,
            "pn_w": 1 + 0.1 * torch.randn(W, generator=g), "pn_b": 0.1 * torch.randn(W, generator=g),
            "wo_w": 0.02 * torch.randn(W, W, generator=g), "wo_b": 0.02 * torch.randn(W, generator=g)}


def run(inp, dout, dtype, eps=1e-6):
    leaves = {k: (inp[k].to(DEV, dtype) if k == "XQW" else inp[k].to(DEV)).detach().requires_grad_(True)
              for k in ARGS}
    out = post_norm_wo(*(leaves[k] for k in ARGS), eps)
    (out.float() * dout.to(DEV, dtype).float()).sum().backward()
    return out, {k: leaves[k].grad for k in ARGS}


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(2, 4, 3, 16, 64), (1, 2, 2, 16, 64), (3, 5, 2, 8, 16), (1, 8, 4, 16, 64),
                                   (1, 16, 1, 16, 64)])
def test_epilogue_matches_oracle(dtype, shape):
    """Widths 256, 128, 80 (a ragged last chunk), 512 and 1024 (16-bit) / 512 (fp32 limit)."""
    B, NH, NC, CS, F = shape
    if dtype == torch.float32 and NH * F > 512:
        pytest.skip("fp32 rows are limited to 512 columns")
    inp = inputs(B, NH, NC, CS, F, seed=NH * F + NC)
    dout = torch.randn(B, NC * CS, NH * F, generator=torch.Generator().manual_seed(7))
    out, grads = run(inp, dout, dtype)
    od = {k: (v.to(dtype) if k == "XQW" else v).double() for k, v in inp.items()}
    rg, rout = O.post_norm_wo_grads(od, dout.to(dtype).double())
    tol = TOL[dtype]
    assert out.dtype == dtype
    assert_close("out", out, rout, tol)
    for k in ARGS:
        assert_close("grad " + k, grads[k], rg[k], tol)


def test_epilogue_matches_reference_golden():
    inp, g = load_golden("epilogue")
    out, grads = run(inp, g["dout"], torch.float32, float(g["eps"]))
    assert_close("out", out, g["out"], TOL[torch.float32])
    for k in ARGS:
        assert_close("grad " + k, grads[k], g["grad_" + k], TOL[torch.float32])


def test_output_epilogue_reads_a_layer():
    inp = {k: v.to(DEV) for k, v in inputs(2, 4, 2, 16, 64, seed=1).items()}
    layer = torch.nn.Module()
    layer.post_norm = torch.nn.LayerNorm(256, eps=1e-6).to(DEV)
    layer.wo = torch.nn.Linear(256, 256).to(DEV)
    got = output_epilogue(layer, inp["XQW"])
    want = post_norm_wo(inp["XQW"], layer.post_norm.weight, layer.post_norm.bias, layer.wo.weight, layer.wo.bias)
    assert torch.allclose(got, want)
    ref = layer.wo(layer.post_norm(inp["XQW"].permute(0, 2, 3, 1, 4).reshape(2, 32, 256)))
    assert_close("module", got, ref, 1e-4)
