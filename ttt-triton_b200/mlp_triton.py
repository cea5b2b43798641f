"""Drop-in for the reference's ``mlp_triton.TritonMLP`` (mlp_triton.py:12-468).

    XQW, W1_memo, b1_memo, W2_memo, b2_memo = TritonMLP.apply(
        ttt_norm_weight [NH,F], ttt_norm_bias [NH,F],
        W1_init [B,NH,F,FF], b1_init [B,NH,1,FF], W2_init [B,NH,FF,F], b2_init [B,NH,1,F],
        XQ, XV, XK [B,NH,NC,CS,F], eta [B,NH,NC,CS,CS],
        checkpoint_group_size, memo_segment_size)

XQW is [B,NH,NC,CS,F] in XQ's dtype. The memo states are fp32 [B,NH,NS,...] with
NS = ceil(NC / memo_segment_size), holding the inner state AFTER mini-batch i for each
i % memo_segment_size == 0 (kernels/mlp_forward.py:193-226); they are
non-differentiable (mlp_triton.py:196), and backward receives None for them (no zero
tensors are materialised). Backward returns the twelve gradients of mlp_triton.py:338-351
(LN gradients summed over the batch, full d_eta): the activations' in XQ's dtype, the
parameters' (ttt_norm_weight/bias, W1/b1/W2/b2_init) in each parameter's own dtype. The
reference casts the parameter gradients to XQ's dtype as well, which autograd then casts
back to the parameter's dtype; for fp32 parameters under 16-bit activations that is a
rounding of the gradient (and two copies) which this path skips.
"""

from __future__ import annotations

import torch

import _core
from _sharding import HEAD, LN, local_map


def _forward_core(ctx, ttt_norm_weight, ttt_norm_bias, W1_init, b1_init, W2_init, b2_init, XQ, XV, XK, eta,
                  checkpoint_group_size, memo_segment_size):
    ckpt = int(checkpoint_group_size)
    XQW, last, ck, memo, zs = _core.mlp_forward(
        ttt_norm_weight, ttt_norm_bias, W1_init, b1_init, W2_init, b2_init, XQ, XV, XK, eta, ckpt, memo_segment_size,
        for_backward=any(ctx.needs_input_grad),
    )
    ctx.ckpt = ckpt
    ctx.param_dtypes = (ttt_norm_weight.dtype, ttt_norm_bias.dtype, W1_init.dtype, b1_init.dtype, W2_init.dtype,
                        b2_init.dtype)
    if ck is not None:
        ctx.save_for_backward(XQ, XV, XK, eta, ttt_norm_weight, ttt_norm_bias, *ck, *zs, last[0], last[2])
    ctx.mark_non_differentiable(*memo)
    ctx.set_materialize_grads(False)
    return (XQW, *memo)


def _backward_core(ctx, grad_XQW):
    XQ, XV, XK, eta, ln_w, ln_b, W1c, b1c, W2c, b2c, Z1, Z2, Z1b, Z2b, W1l, W2l = ctx.saved_tensors
    if grad_XQW is None:  # only the (non-differentiable) memo states were used
        grad_XQW = torch.zeros(XQ.shape, device=XQ.device, dtype=XQ.dtype)
    d_ln_w, d_ln_b, dW1, db1, dW2, db2, dXQ, dXV, dXK, deta = _core.mlp_backward(
        ln_w, ln_b, (W1c, b1c, W2c, b2c), XQ, XV, XK, eta, grad_XQW, ctx.ckpt,
        saved=(Z1, Z2, Z1b, Z2b), W1_last=W1l, W2_last=W2l,
    )
    dt = ctx.param_dtypes
    return (
        d_ln_w.sum(0).reshape(ln_w.shape).to(dt[0]),
        d_ln_b.sum(0).reshape(ln_b.shape).to(dt[1]),
        dW1.to(dt[2]), db1.to(dt[3]), dW2.to(dt[4]), db2.to(dt[5]),
        dXQ, dXV, dXK, deta,
        None, None,
    )


_forward_sharded = local_map(
    _forward_core,
    in_placements=(None, LN, LN, HEAD, HEAD, HEAD, HEAD, HEAD, HEAD, HEAD, HEAD, None, None),
    out_placements=(HEAD, HEAD, HEAD, HEAD, HEAD),
)
_backward_sharded = local_map(
    _backward_core,
    in_placements=(None, HEAD),
    out_placements=(LN, LN, HEAD, HEAD, HEAD, HEAD, HEAD, HEAD, HEAD, HEAD, None, None),
)


class TritonMLP(torch.autograd.Function):
    sharded_mode = False

    @staticmethod
    def forward(ctx, ttt_norm_weight, ttt_norm_bias, W1_init, b1_init, W2_init, b2_init, XQ_batch, XV_batch,
                XK_batch, eta_batch, checkpoint_group_size, memo_segment_size):
        core = _forward_sharded if TritonMLP.sharded_mode else _forward_core
        return core(ctx, ttt_norm_weight, ttt_norm_bias, W1_init, b1_init, W2_init, b2_init, XQ_batch, XV_batch,
                    XK_batch, eta_batch, checkpoint_group_size, memo_segment_size)

    @staticmethod
    def backward(ctx, grad_L_XQW_batch, *unused):
        core = _backward_sharded if TritonMLP.sharded_mode else _backward_core
        return core(ctx, grad_L_XQW_batch)
