"""GPU: the allocation-free TTT-Linear backward matches the caller-scratch backward.

``ttt_linear_bwd_noalloc`` is for callers that cannot allocate device memory where they
enqueue work, such as an inference-engine plugin that is only handed pre-sized buffers
or a service that fixes its device-memory budget at start-up. It takes its scratch from
a fixed 16 MiB array inside the library. This test calls it through the C ABI twice in a
row, with different inputs, and compares each result with ``ttt_linear_bwd`` given an
explicit scratch buffer, at the parity tolerance of the inputs' dtype. The file name
makes pytest collect it last.
"""

import pytest
import torch

import _core
import synthetic as S
from _lib import check, dtype_code, lib, ptr, stream_of
from helpers import TOL, assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"
NAMES = ("ln_w", "ln_b", "W1", "b1", "XQ", "XV", "XK", "eta")


def _case(B, NH, NC, F, dtype, seed):
    d = S.perturb_params(S.make_linear_inputs(B, NH, NC, 16, F, seed=seed), seed=seed + 5)
    d = {k: (v.to(DEV, dtype) if k in ("XQ", "XK", "XV", "eta") else v.to(DEV)) for k, v in d.items()}
    dO = S.make_upstream((B, NH, NC, 16, F), seed=seed + 1).to(DEV, dtype)
    return d, dO


def _noalloc_backward(d, W_ckpt, b_ckpt, dO, ckpt):
    B, NH, NC, CS, F = d["XQ"].shape
    f32 = dict(device=DEV, dtype=torch.float32)
    out = {
        "ln_w": torch.empty(B, NH, F, **f32), "ln_b": torch.empty(B, NH, F, **f32),
        "W1": torch.empty(B, NH, F, F, **f32), "b1": torch.empty(B, NH, 1, F, **f32),
        "XQ": torch.empty_like(d["XQ"]), "XV": torch.empty_like(d["XQ"]), "XK": torch.empty_like(d["XQ"]),
        "eta": torch.empty_like(d["eta"]),
    }
    rc = lib.ttt_linear_bwd_noalloc(
        B, NH, NC, CS, F, ckpt,
        ptr(d["ln_w"]), ptr(d["ln_b"]), dtype_code(d["ln_w"]),
        ptr(W_ckpt), ptr(b_ckpt),
        ptr(d["XQ"]), dtype_code(d["XQ"]), ptr(d["XV"]), dtype_code(d["XV"]), ptr(d["XK"]), dtype_code(d["XK"]),
        ptr(d["eta"]), dtype_code(d["eta"]),
        ptr(dO), dtype_code(dO),
        ptr(out["ln_w"]), ptr(out["ln_b"]), ptr(out["W1"]), ptr(out["b1"]),
        ptr(out["XQ"]), ptr(out["XV"]), ptr(out["XK"]), ptr(out["eta"]), dtype_code(out["XQ"]),
        stream_of(d["XQ"]),
    )
    check(rc, "ttt_linear_bwd_noalloc")
    return out


@pytest.mark.parametrize("dtype,F", [(torch.float32, 32), (torch.bfloat16, 64)])
def test_noalloc_backward_matches_scratch_backward_twice(dtype, F):
    tol = TOL[dtype]
    for call, (B, NH, NC, ckpt, seed) in enumerate(((2, 3, 10, 4, 40), (1, 2, 7, 3, 50))):
        d, dO = _case(B, NH, NC, F, dtype, seed)
        _, _, _, W_ckpt, b_ckpt, _ = _core.linear_forward(*(d[k] for k in NAMES), ckpt)
        ref = dict(zip(("ln_w", "ln_b", "W1", "b1", "XQ", "XV", "XK", "eta"),
                       _core.linear_backward(d["ln_w"], d["ln_b"], W_ckpt, b_ckpt, d["XQ"], d["XV"], d["XK"],
                                             d["eta"], dO, ckpt)))
        got = _noalloc_backward(d, W_ckpt, b_ckpt, dO, ckpt)
        torch.cuda.synchronize()
        for k in ref:
            assert_close(f"call {call + 1}: d{k}", got[k], ref[k], tol)
