"""Output epilogue of the TTT layer on the sm_100a kernels: the permute of the scan output to
token order (TTTMLP.ttt, ttt_layer.py:563-564; TTTLinear.ttt :405,420), post_norm (:349) and
wo (:350).

The reference copies the permuted scan output, layer-normalises it into a second copy and
projects that. Here one kernel reads the scan output in its [B, NH, NC, CS, F] layout and
writes the normalised rows; wo is one library GEMM with its bias fused. Backward: two
library GEMMs for wo and one kernel that writes d XQW straight back into the scan layout.
A maintainer switches the layer over by returning the scan output in kernel layout from
ttt() and replacing lines 349-350 of TTTBase.forward with

    hidden_states = epilogue.output_epilogue(self, XQW_batch)
"""

from __future__ import annotations

import torch

import _core


class PostNormWo(torch.autograd.Function):
    @staticmethod
    def forward(ctx, XQW, pn_w, pn_b, wo_w, wo_b, eps):
        B, NH, NC, CS, F = XQW.shape
        W = NH * F
        Y = _core.post_norm_forward(XQW, pn_w, pn_b, eps)  # [B * L, W], token order
        out = torch.addmm(wo_b, Y, wo_w.t())
        ctx.eps = float(eps)
        ctx.pn_dtypes = (pn_w.dtype, pn_b.dtype)
        ctx.save_for_backward(XQW, Y, pn_w, pn_b, wo_w)
        return out.view(B, NC * CS, W)

    @staticmethod
    def backward(ctx, dout):
        XQW, Y, pn_w, pn_b, wo_w = ctx.saved_tensors
        d2 = dout.reshape(Y.shape)
        if not d2.is_contiguous():
            d2 = d2.contiguous()
        d2 = d2.to(Y.dtype)
        dY = torch.mm(d2, wo_w)
        dwo_w = torch.mm(d2.t(), Y)
        # the kernel also sums d out over tokens: the wo bias gradient
        dXQW, dpn_w, dpn_b, dwo_b = _core.post_norm_backward(XQW, pn_w, pn_b, ctx.eps, dY, d2)
        return dXQW, dpn_w.to(ctx.pn_dtypes[0]), dpn_b.to(ctx.pn_dtypes[1]), dwo_w, dwo_b.to(wo_w.dtype), None


def post_norm_wo(XQW_batch, post_norm_weight, post_norm_bias, wo_weight, wo_bias, eps=1e-6):
    """wo(post_norm(XQW_batch in token order)) -> [B, L, W] in XQW_batch's dtype.
    XQW_batch [B, NH, NC, CS, F] (the scan's layout); post_norm_* [W]; wo_* [W, W], [W]."""
    if XQW_batch.dim() != 5:
        raise ValueError(f"XQW_batch must be [B, NH, NC, CS, F], got {tuple(XQW_batch.shape)}")
    dt = XQW_batch.dtype
    return PostNormWo.apply(XQW_batch, post_norm_weight, post_norm_bias, wo_weight.to(dt), wo_bias.to(dt), eps)


def output_epilogue(layer, XQW_batch):
    """Drop-in for the permute of ttt() plus ``self.wo(self.post_norm(...))`` of a TTTBase
    layer (ttt_layer.py:349-350): reads layer.post_norm (weight, bias, eps) and layer.wo."""
    pn = layer.post_norm
    return post_norm_wo(XQW_batch, pn.weight, pn.bias, layer.wo.weight, layer.wo.bias, pn.eps)
