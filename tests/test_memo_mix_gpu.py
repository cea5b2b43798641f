"""GPU parity of the fused memo-state mixing (ttt_layer.py:503-559) against the oracle."""

import pytest
import torch

import _core
import synthetic as S
import ttt_oracle as O
from helpers import assert_close, oracle_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"
SCAN = ("ln_w", "ln_b", "W1", "b1", "W2", "b2", "XQ", "XV", "XK", "eta")


def make(B, NH, NC, M, dtype, seed, FF=256):
    d = S.perturb_params(S.make_mlp_inputs(B, NH, NC, 16, 64, FF, seed=seed), seed=seed + 1)
    d = {k: (v.to(dtype) if k in ("XQ", "XV", "XK", "eta") else v) for k, v in d.items()}
    od = oracle_inputs(d)
    r = O.mlp_scan(*(od[k] for k in SCAN), 1, M)
    g = torch.Generator().manual_seed(seed + 2)
    XU = (torch.randn(B, NH, NC, 16, 64, generator=g)).to(dtype)
    inp = {"XQW": r["XQW"].to(dtype), "XQ": d["XQ"], "XK": d["XK"], "XU": XU,
           "W1_memo": r["W1_memo"].float(), "b1_memo": r["b1_memo"].float(), "W2_memo": r["W2_memo"].float(),
           "b2_memo": r["b2_memo"].float(), "ln_w": d["ln_w"], "ln_b": d["ln_b"]}
    return inp


ORDER = ("XQW", "XQ", "XK", "XU", "W1_memo", "b1_memo", "W2_memo", "b2_memo", "ln_w", "ln_b")


@pytest.mark.parametrize("FF", [256, 64])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(1, 2, 7, 2), (1, 1, 40, 16), (2, 1, 9, 3), (2, 2, 21, 2), (1, 1, 40, 2)])
def test_memo_mix_matches_oracle(dtype, shape, FF):
    """Forward and gradients (XQW, XU, XK) of the fused kernels for the 256-wide and the F x F
    inner MLP, including segments of 256 tokens (two 128-token tiles), a ragged last segment,
    the config-4 layer's 11 segments of 2 mini-batches (F x F: two CTAs per SM) and 20
    segments (F x F: more memo states than the two-CTA kernel holds, the one-CTA kernel)."""
    B, NH, NC, M = shape
    inp = make(B, NH, NC, M, dtype, seed=NC + M, FF=FF)
    dO = S.make_upstream((B, NH, NC, 16, 64), seed=3).to(dtype)
    from kernels.mlp_memo_mix import fused_envelope, mlp_memo_mix

    assert fused_envelope(inp["XQW"], inp["W1_memo"], M)

    leaves = {k: (v.to(DEV).requires_grad_(k in ("XQW", "XU", "XK")) if v.is_floating_point() else v.to(DEV))
              for k, v in inp.items()}
    out = mlp_memo_mix(*(leaves[k] for k in ORDER), M)
    out.backward(dO.to(DEV))
    ref_g, ref = O.memo_mix_grads({k: v.double() for k, v in inp.items()}, dO.double(), M)
    assert out.dtype == dtype and out.shape == inp["XQW"].shape
    assert_close("out", out, ref, 2e-2)
    for k in ("XQW", "XU", "XK"):
        assert_close("d" + k, leaves[k].grad, ref_g[k], 2e-2)
    # segment 0 passes through unchanged
    assert torch.equal(out[:, :, :M].cpu(), inp["XQW"][:, :, :M])


def test_memo_mix_rejects_unsupported_shapes_and_no_wait_gave_up():
    import _lib

    inp = make(1, 1, 4, 2, torch.bfloat16, seed=7)
    dev = {k: v.to(DEV) for k, v in inp.items()}
    with pytest.raises(ValueError, match="memo_segment_size"):
        _core.memo_mix_forward(*(dev[k] for k in ORDER), 0)
    _lib.device_status()
    _core.memo_mix_forward(*(dev[k] for k in ORDER), 2)
    assert _lib.device_status() == 0


@pytest.mark.parametrize("FF", [256, 64])
def test_backward_reuses_the_forward_scratch(FF):
    """A backward given the forward's scratch (prepared operands and summaries) gives the
    same gradients as one that prepares them itself."""
    inp = make(2, 1, 9, 2, torch.bfloat16, seed=11, FF=FF)
    dev = {k: v.to(DEV) for k, v in inp.items()}
    dO = S.make_upstream((2, 1, 9, 16, 64), seed=12).to(DEV, torch.bfloat16)
    out, scratch = _core.memo_mix_forward(*(dev[k] for k in ORDER), 2, return_scratch=True)
    assert torch.equal(out, _core.memo_mix_forward(*(dev[k] for k in ORDER), 2))
    fresh = _core.memo_mix_backward(*(dev[k] for k in ORDER), 2, dO)
    reused = _core.memo_mix_backward(*(dev[k] for k in ORDER), 2, dO, scratch=scratch)
    assert torch.equal(fresh[0], reused[0]) and torch.equal(fresh[1], reused[1])
    assert torch.allclose(fresh[2].float(), reused[2].float(), rtol=1e-2, atol=1e-6)  # d summary atomics
