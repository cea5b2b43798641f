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
        out, scratch = _core.memo_mix_forward(XQW, XQ, XK, XU, W1_memo, b1_memo, W2_memo, b2_memo, ln_w, ln_b,
                                              memo_segment_size, return_scratch=True)
        ctx.memo_segment_size = int(memo_segment_size)
        ctx.scratch = scratch  # prepared memo operands and summaries, reused by the backward
        ctx.save_for_backward(XQW, XQ, XK, XU, W1_memo, b1_memo, W2_memo, b2_memo, ln_w, ln_b)
        return out

    @staticmethod
    def backward(ctx, dOut):
        XQW, XQ, XK, XU, W1_memo, b1_memo, W2_memo, b2_memo, ln_w, ln_b = ctx.saved_tensors
        dXQW, dXU, dXK = _core.memo_mix_backward(XQW, XQ, XK, XU, W1_memo, b1_memo, W2_memo, b2_memo, ln_w, ln_b,
                                                 ctx.memo_segment_size, dOut, scratch=ctx.scratch)
        ctx.scratch = None
        return dXQW, None, dXK, dXU, None, None, None, None, None, None, None


def fused_envelope(XQW_batch, W1_memo, memo_segment_size):
    """True when the fused mixing kernels take these shapes: CS = 16, F = 64, an inner width
    of 256 or 64 (the layer's F x F MLP), 16-bit activations, at most 64 memo segments
    (ttt_memo_mix.cu)."""
    B, NH, NC, CS, F = XQW_batch.shape
    NS = -(-NC // int(memo_segment_size))
    return (CS == 16 and F == 64 and W1_memo.shape[-1] in (256, 64) and NS <= 64
            and XQW_batch.dtype in (torch.bfloat16, torch.float16))


def memo_mix_segments(XQW_batch, XQ, XK, XU, W1_memo, b1_memo, W2_memo, b2_memo, ttt_norm_weight, ttt_norm_bias,
                      memo_segment_size):
    """The segment loop of ttt_layer.py:503-559 as the reference runs it, with every cached
    read-out on this library's ``ttt_mlp_cached_readout`` kernel: the path for shapes outside
    the fused kernels (e.g. the layer's F x F inner MLP). Differentiable in XQW, XU and XK
    through the torch ops (the cached read-outs carry no gradient, :542); the mixing follows
    the reference's dtypes (gamma cast to the activation dtype, fp32 cached sum, :536-556)."""
    B, NH, NC, CS, F = XQW_batch.shape
    M = int(memo_segment_size)
    dt = XQW_batch.dtype
    out, cached = [], []
    for i in range(-(-NC // M)):
        s0, s1 = i * M, min((i + 1) * M, NC)
        XQ_seg, XU_seg, XQW_seg = XQ[:, :, s0:s1], XU[:, :, s0:s1], XQW_batch[:, :, s0:s1]
        summary_cur = XK[:, :, s0:s1].mean(dim=(2, 3))
        if i == 0:
            cached.append(summary_cur.detach())
            out.append(XQW_seg)
            continue
        sims = [(XU_seg * summ[:, :, None, None, :]).sum(dim=-1) for summ in cached]
        sims.append((XU_seg * summary_cur[:, :, None, None, :]).sum(dim=-1))
        gamma = torch.softmax(torch.stack(sims, dim=-1), dim=-1)
        seg = gamma[..., -1:].to(dt) * XQW_seg
        cached_sum = torch.zeros(seg.shape, device=seg.device, dtype=torch.float32)
        XQ_c = XQ_seg.contiguous()
        for j in range(i):
            with torch.no_grad():
                delta = _core.mlp_cached_readout(XQ_c, W1_memo[:, :, j], b1_memo[:, :, j], W2_memo[:, :, j],
                                                 b2_memo[:, :, j], ttt_norm_weight, ttt_norm_bias)
            cached_sum = cached_sum + gamma[..., j:j + 1].to(torch.float32) * delta
        out.append(seg + cached_sum.to(dt))
        cached.append(summary_cur.detach())
    return torch.cat(out, dim=2)


def mlp_memo_mix(XQW_batch, XQ, XK, XU, W1_memo, b1_memo, W2_memo, b2_memo, ttt_norm_weight, ttt_norm_bias,
                 memo_segment_size):
    """Mixed layer output [B, NH, NC, CS, F]: the fused kernels inside their envelope, else
    the segment loop on the cached read-out kernel."""
    if fused_envelope(XQW_batch, W1_memo, memo_segment_size):
        return MemoMix.apply(XQW_batch, XQ, XK, XU, W1_memo, b1_memo, W2_memo, b2_memo, ttt_norm_weight,
                             ttt_norm_bias, memo_segment_size)
    return memo_mix_segments(XQW_batch, XQ, XK, XU, W1_memo, b1_memo, W2_memo, b2_memo, ttt_norm_weight,
                             ttt_norm_bias, memo_segment_size)
