"""``ttt_mlp`` with the signature and output layout of ops/ttt_mlp.py:70-99.

    XQW = ttt_mlp(XK, XQ, XV, eta, ttt_norm_weight, ttt_norm_bias, W1_init, b1_init,
                  W2_init, b2_init, checkpoint_group_size)   # -> [B, NC, CS, NH, F]
"""

from __future__ import annotations

import torch

import _core


class _MLPScan(torch.autograd.Function):
    """TTT-MLP scan without memo outputs (the ops path never reads them).

    Gradients come back in each input's own dtype, as autograd over the reference's ops/
    path returns them: the activations' in XQ's dtype, the parameters' (ln_w, ln_b, W1,
    b1, W2, b2) in the parameter's dtype (fp32 parameters get fp32 gradients), the same
    rule as mlp_triton.TritonMLP."""

    @staticmethod
    def forward(ctx, ln_w, ln_b, W1, b1, W2, b2, XQ, XV, XK, eta, ckpt):
        XQW, last, ck, _, zs = _core.mlp_forward(ln_w, ln_b, W1, b1, W2, b2, XQ, XV, XK, eta, ckpt, None,
                                                 for_backward=any(ctx.needs_input_grad))
        ctx.ckpt = ckpt
        ctx.param_dtypes = (ln_w.dtype, ln_b.dtype, W1.dtype, b1.dtype, W2.dtype, b2.dtype)
        if ck is not None:
            ctx.save_for_backward(XQ, XV, XK, eta, ln_w, ln_b, *ck, *zs, last[0], last[2])
        return XQW

    @staticmethod
    def backward(ctx, grad):
        XQ, XV, XK, eta, ln_w, ln_b, W1c, b1c, W2c, b2c, Z1, Z2, Z1b, Z2b, W1l, W2l = ctx.saved_tensors
        d_ln_w, d_ln_b, dW1, db1, dW2, db2, dXQ, dXV, dXK, deta = _core.mlp_backward(
            ln_w, ln_b, (W1c, b1c, W2c, b2c), XQ, XV, XK, eta, grad, ctx.ckpt,
            saved=(Z1, Z2, Z1b, Z2b), W1_last=W1l, W2_last=W2l,
        )
        dt = ctx.param_dtypes
        return (d_ln_w.sum(0).reshape(ln_w.shape).to(dt[0]), d_ln_b.sum(0).reshape(ln_b.shape).to(dt[1]),
                dW1.to(dt[2]), db1.to(dt[3]), dW2.to(dt[4]), db2.to(dt[5]), dXQ, dXV, dXK, deta, None)


def ttt_mlp(XK, XQ, XV, eta, ttt_norm_weight, ttt_norm_bias, W1_init, b1_init, W2_init, b2_init,
            checkpoint_group_size):
    NC = XQ.shape[2]
    ckpt = int(checkpoint_group_size)
    ckpt = NC if ckpt <= 0 else min(ckpt, NC)
    out = _MLPScan.apply(ttt_norm_weight, ttt_norm_bias, W1_init, b1_init, W2_init, b2_init, XQ, XV, XK, eta, ckpt)
    return out.permute(0, 2, 3, 1, 4)
