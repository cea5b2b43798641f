"""Memo-state mixing of the TTT-MLP layer's output, fused (the segment loop of
ttt_layer.py:503-559).

The reference mixes, for every memo segment i >= 1, the online output with the cached
read-outs of all earlier memo states: one ``mlp_cached_readout_triton`` launch per
(segment, earlier state) pair from Python, O(NS^2) launches. Here the whole loop is one
launch sequence on the sm_100a tensor cores:

    XQW_batch = mlp_memo_mix(XQW_batch, inputs["XQ"], inputs["XK"], inputs["XU"],
                             W1_memo, b1_memo, W2_memo, b2_memo,
                             self.ttt_norm_weight, self.ttt_norm_bias, memo_segment_size)

replaces lines 503-559 of ``TTTMLP.ttt`` (XQW_batch and the inputs in kernel layout
[B, NH, NC, CS, F], memo states as ``TritonMLP`` returns them). Gradients flow into XQW,
XU and XK (through the current segment's summary), exactly as in the reference; the cached
read-outs and earlier summaries carry none.
"""

from __future__ import annotations

import torch

import _core


class MemoMix(torch.autograd.Function):
    @staticmethod
    def forward(ctx, XQW, XQ, XK, XU, W1_memo, b1_memo, W2_memo, b2_memo, ln_w, ln_b, memo_segment_size):
        out = _core.memo_mix_forward(XQW, XQ, XK, XU, W1_memo, b1_memo, W2_memo, b2_memo, ln_w, ln_b,
                                     memo_segment_size)
        ctx.memo_segment_size = int(memo_segment_size)
        ctx.save_for_backward(XQW, XQ, XK, XU, W1_memo, b1_memo, W2_memo, b2_memo, ln_w, ln_b)
        return out

    @staticmethod
    def backward(ctx, dOut):
        XQW, XQ, XK, XU, W1_memo, b1_memo, W2_memo, b2_memo, ln_w, ln_b = ctx.saved_tensors
        dXQW, dXU, dXK = _core.memo_mix_backward(XQW, XQ, XK, XU, W1_memo, b1_memo, W2_memo, b2_memo, ln_w, ln_b,
                                                 ctx.memo_segment_size, dOut)
        return dXQW, None, dXK, dXU, None, None, None, None, None, None, None


def mlp_memo_mix(XQW_batch, XQ, XK, XU, W1_memo, b1_memo, W2_memo, b2_memo, ttt_norm_weight, ttt_norm_bias,
                 memo_segment_size):
    return MemoMix.apply(XQW_batch, XQ, XK, XU, W1_memo, b1_memo, W2_memo, b2_memo, ttt_norm_weight,
                         ttt_norm_bias, memo_segment_size)
