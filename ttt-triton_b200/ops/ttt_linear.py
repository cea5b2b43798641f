"""``ttt_linear`` with the signature and output layout of ops/ttt_linear.py:57-84.

    XQW = ttt_linear(XK, XQ, XV, eta, ttt_norm_weight, ttt_norm_bias, W1_init, b1_init,
                     checkpoint_group_size)            # -> [B, NC, CS, NH, F]

Differentiable w.r.t. every tensor argument. checkpoint_group_size <= 0 means one group
(the reference's ``scan`` without checkpointing); it changes memory use, not results.
"""

from __future__ import annotations

from linear_triton import TritonLinear


def ttt_linear(XK, XQ, XV, eta, ttt_norm_weight, ttt_norm_bias, W1_init, b1_init, checkpoint_group_size):
    NC = XQ.shape[2]
    ckpt = int(checkpoint_group_size)
    ckpt = NC if ckpt <= 0 else min(ckpt, NC)
    out = TritonLinear.apply(ttt_norm_weight, ttt_norm_bias, W1_init, b1_init, XQ, XV, XK, eta, ckpt)
    return out.permute(0, 2, 3, 1, 4)
