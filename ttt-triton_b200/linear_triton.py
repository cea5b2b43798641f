"""Drop-in for the reference's ``linear_triton.TritonLinear`` (linear_triton.py:12-362).

Same autograd signature and output layout, computed by the sm_100a kernels of
libttt_b200.so (no Triton):

    XQW = TritonLinear.apply(ttt_norm_weight [NH,F], ttt_norm_bias [NH,F],
                             W1_init [B,NH,F,F], b1_init [B,NH,1,F],
                             XQ, XV, XK [B,NH,NC,CS,F], eta [B,NH,NC,CS,CS],
                             checkpoint_group_size)

XQW is [B,NH,NC,CS,F] in XQ's dtype (computed in fp32). Backward returns the ten
gradients of linear_triton.py:254-265: the LN parameter gradients summed over the batch,
dW1, db1 (each in its parameter's dtype; the reference casts them to XQ's dtype, which
autograd casts back, a rounding this path skips for fp32 parameters), dXQ, dXV, dXK, the
full dual-form d_eta (in XQ's dtype), None, None.
``TritonLinear.sharded_mode`` selects the head-sharded DTensor entry, as in the reference.
"""

from __future__ import annotations

import torch

import _core
from _sharding import HEAD, LN, local_map


def _forward_core(ctx, ttt_norm_weight, ttt_norm_bias, W1_init, b1_init, XQ, XV, XK, eta, checkpoint_group_size):
    ckpt = int(checkpoint_group_size)
    train = any(ctx.needs_input_grad)
    XQW, W_last, b_last, W_ckpt, b_ckpt, Z = _core.linear_forward(
        ttt_norm_weight, ttt_norm_bias, W1_init, b1_init, XQ, XV, XK, eta, ckpt, for_backward=train
    )
    ctx.ckpt = ckpt
    ctx.param_dtypes = (ttt_norm_weight.dtype, ttt_norm_bias.dtype, W1_init.dtype, b1_init.dtype)
    if train:
        ctx.save_for_backward(XQ, XV, XK, eta, ttt_norm_weight, ttt_norm_bias, W_ckpt, b_ckpt, Z, W_last, b_last)
    return XQW


def _backward_core(ctx, grad_XQW):
    XQ, XV, XK, eta, ln_w, ln_b, W_ckpt, b_ckpt, Z, W_last, b_last = ctx.saved_tensors
    d_ln_w, d_ln_b, dW1, db1, dXQ, dXV, dXK, deta = _core.linear_backward(
        ln_w, ln_b, W_ckpt, b_ckpt, XQ, XV, XK, eta, grad_XQW, ctx.ckpt, Z=Z, W_last=W_last, b_last=b_last
    )
    dt = ctx.param_dtypes
    return (
        d_ln_w.sum(0).reshape(ln_w.shape).to(dt[0]),
        d_ln_b.sum(0).reshape(ln_b.shape).to(dt[1]),
        dW1.to(dt[2]),
        db1.to(dt[3]),
        dXQ,
        dXV,
        dXK,
        deta,
        None,
        None,
    )


_forward_sharded = local_map(
    _forward_core,
    in_placements=(None, LN, LN, HEAD, HEAD, HEAD, HEAD, HEAD, HEAD, None),
    out_placements=(HEAD,),
)
_backward_sharded = local_map(
    _backward_core,
    in_placements=(None, HEAD),
    out_placements=(LN, LN, HEAD, HEAD, HEAD, HEAD, HEAD, HEAD, None, None),
)


class TritonLinear(torch.autograd.Function):
    sharded_mode = False

    @staticmethod
    def forward(ctx, ttt_norm_weight, ttt_norm_bias, W1_init, b1_init, XQ_batch, XV_batch, XK_batch, eta_batch,
                checkpoint_group_size) -> torch.Tensor:
        core = _forward_sharded if TritonLinear.sharded_mode else _forward_core
        return core(ctx, ttt_norm_weight, ttt_norm_bias, W1_init, b1_init, XQ_batch, XV_batch, XK_batch, eta_batch,
                    checkpoint_group_size)

    @staticmethod
    def backward(ctx, grad_L_XQW_batch):
        core = _backward_sharded if TritonLinear.sharded_mode else _backward_core
        return core(ctx, grad_L_XQW_batch)
