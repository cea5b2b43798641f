"""Drop-in for the reference's ``mlp_triton_back.TritonMLP`` (mlp_triton_back.py:12-422).

The F x F TTT-MLP (W1, W2 both [B,NH,F,F]) without memo outputs:

    XQW = TritonMLP.apply(ttt_norm_weight, ttt_norm_bias, W1_init, b1_init, W2_init, b2_init,
                          XQ, XV, XK, eta, checkpoint_group_size)

The reference module launches its kernels with an argument list that no longer matches
them, so it cannot run as shipped; this one runs the sm_100a MLP kernels with FF = F.
Backward returns the twelve gradients of mlp_triton_back.py:301-314, the parameters' in
each parameter's own dtype (the reference casts them to XQ's dtype first), the
activations' in XQ's dtype.
"""

from __future__ import annotations

import torch

import _core
from _sharding import HEAD, LN, local_map


def _forward_core(ctx, ttt_norm_weight, ttt_norm_bias, W1_init, b1_init, W2_init, b2_init, XQ, XV, XK, eta,
                  checkpoint_group_size):
    F = XQ.shape[-1]
    if W1_init.shape[-1] != F or W2_init.shape[-2] != F:
        raise ValueError(f"mlp_triton_back.TritonMLP is the F x F MLP; got W1 {tuple(W1_init.shape)}, "
                         f"W2 {tuple(W2_init.shape)} for F = {F}")
    ckpt = int(checkpoint_group_size)
    XQW, last, ck, _, zs = _core.mlp_forward(
        ttt_norm_weight, ttt_norm_bias, W1_init, b1_init, W2_init, b2_init, XQ, XV, XK, eta, ckpt, None,
        for_backward=any(ctx.needs_input_grad),
    )
    ctx.ckpt = ckpt
    ctx.param_dtypes = (ttt_norm_weight.dtype, ttt_norm_bias.dtype, W1_init.dtype, b1_init.dtype, W2_init.dtype,
                        b2_init.dtype)
    if ck is not None:
        ctx.save_for_backward(XQ, XV, XK, eta, ttt_norm_weight, ttt_norm_bias, *ck, *zs, last[0], last[2])
    return XQW


def _backward_core(ctx, grad_XQW):
    XQ, XV, XK, eta, ln_w, ln_b, W1c, b1c, W2c, b2c, Z1, Z2, Z1b, Z2b, W1l, W2l = ctx.saved_tensors
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
        None,
    )


_forward_sharded = local_map(
    _forward_core,
    in_placements=(None, LN, LN, HEAD, HEAD, HEAD, HEAD, HEAD, HEAD, HEAD, HEAD, None),
    out_placements=(HEAD,),
)
_backward_sharded = local_map(
    _backward_core,
    in_placements=(None, HEAD),
    out_placements=(LN, LN, HEAD, HEAD, HEAD, HEAD, HEAD, HEAD, HEAD, HEAD, None),
)


class TritonMLP(torch.autograd.Function):
    sharded_mode = False

    @staticmethod
    def forward(ctx, ttt_norm_weight, ttt_norm_bias, W1_init, b1_init, W2_init, b2_init, XQ_batch, XV_batch,
                XK_batch, eta_batch, checkpoint_group_size) -> torch.Tensor:
        core = _forward_sharded if TritonMLP.sharded_mode else _forward_core
        return core(ctx, ttt_norm_weight, ttt_norm_bias, W1_init, b1_init, W2_init, b2_init, XQ_batch, XV_batch,
                    XK_batch, eta_batch, checkpoint_group_size)

    @staticmethod
    def backward(ctx, grad_L_XQW_batch):
        core = _backward_sharded if TritonMLP.sharded_mode else _backward_core
        return core(ctx, grad_L_XQW_batch)
