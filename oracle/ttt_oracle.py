"""CPU oracle for the TTT-Linear / TTT-MLP mini-batch dual-form scan.

TEST INFRASTRUCTURE ONLY. This module is the checker the CUDA path is compared
against; it is never the thing measured or shipped. Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs of
``bench.py`` may import it. The product path (``ttt-triton_b200/``) never imports it
and fails loudly when its CUDA library is missing.

What it restates (reference paths are relative to the Ali-Najar/ttt-triton root):

* ``ln_fwd``             -> ops/ttt_utils.py:4-18   (biased variance, eps 1e-8)
* ``ln_fused_l2_bwd``    -> ops/ttt_utils.py:21-48  (closed-form d/dx of 1/2||LN(x)-t||^2)
* ``gelu_bwd``           -> ops/ttt_utils.py:51-54  (tanh-GELU derivative, truncated constants)
* ``linear_step``        -> ops/ttt_linear.py:8-54  (compute_mini_batch, dual form)
* ``mlp_step``           -> ops/ttt_mlp.py:9-67     (compute_mini_batch, dual form)
* ``ttt_linear``/``ttt_mlp`` -> ops/ttt_linear.py:57-84, ops/ttt_mlp.py:70-99 and the
  scan driver utils.py:126-161. Activation checkpointing there changes memory only,
  not values, so the oracle runs the plain loop.
* checkpoint / memo / final-state side outputs -> kernels/linear_forward.py:54-73,147-148
  and kernels/mlp_forward.py:83-117,193-237 (state at the START of every checkpoint
  group; memo = state AFTER mini-batch i for i % memo_segment_size == 0).
* ``mlp_cached_readout`` -> kernels/mlp_cached_readout.py:7-109,112-143 with the
  (b, h) offsets the kernel intends (its shipped offsets drop b and h, so only the
  (0, 0) slice of the shipped kernel is meaningful; the goldens use B = NH = 1).

Parity is pinned by ``tests/golden/*.npz``, generated from the reference's own
``ops/`` package and Triton kernel (``tests/golden/make_golden.py``) and checked by
``tests/test_oracle.py``. Gradients come from torch autograd through this
restatement, exactly as the reference's ``ops/`` path gets them; ``dual_bwd.py``
holds the hand-derived backward the CUDA kernels implement and is checked against
these autograd gradients.

Everything runs in the dtype of the inputs (the tests use float64).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as Fn

LN_EPS = 1e-8  # ops/ttt_utils.py:4,21
READOUT_EPS = 1e-6  # kernels/mlp_cached_readout.py:99


# --------------------------------------------------------------------------- helpers
def ln_fwd(x, gamma, beta, eps=LN_EPS):
    """LayerNorm forward, biased variance (ops/ttt_utils.py:4-18)."""
    mu = x.mean(dim=-1, keepdim=True)
    var = x.var(dim=-1, keepdim=True, unbiased=False)
    std = torch.sqrt(var + eps)
    return gamma * ((x - mu) / std) + beta


def ln_fused_l2_bwd(x, l2_target, gamma, beta, eps=LN_EPS):
    """Gradient of 1/2 ||LN(x) - target||^2 w.r.t. x (ops/ttt_utils.py:21-48)."""
    D = x.shape[-1]
    mu = x.mean(dim=-1, keepdim=True)
    var = x.var(dim=-1, keepdim=True, unbiased=False)
    std = torch.sqrt(var + eps)
    x_hat = (x - mu) / std
    y = gamma * x_hat + beta
    grad_output = y - l2_target
    grad_x_hat = grad_output * gamma
    return (
        (1.0 / D)
        * (
            D * grad_x_hat
            - grad_x_hat.sum(dim=-1, keepdim=True)
            - x_hat * (grad_x_hat * x_hat).sum(dim=-1, keepdim=True)
        )
        / std
    )


def gelu_bwd(x):
    """tanh-GELU derivative with the reference's truncated constants (ops/ttt_utils.py:51-54)."""
    tanh_out = torch.tanh(0.79788456 * x * (1 + 0.044715 * x * x))
    return 0.5 * x * ((1 - tanh_out * tanh_out) * (0.79788456 + 0.1070322243 * x * x)) + 0.5 * (1 + tanh_out)


def gelu_tanh(x):
    """F.gelu(approximate="tanh") as used by ops/ttt_mlp.py:16,28."""
    return Fn.gelu(x, approximate="tanh")


class _Round(torch.autograd.Function):
    """Rounds a tensor to a 16-bit type in the forward and the gradient reaching it to the
    same type in the backward, keeping the working dtype (float64 in the tests)."""

    @staticmethod
    def forward(ctx, x, dt):
        ctx.dt = dt
        return x.to(dt).to(x.dtype)

    @staticmethod
    def backward(ctx, g):
        return g.to(ctx.dt).to(g.dtype), None


def rounding(dt):
    """The tensor-boundary rounding of a 16-bit activation path: a function that rounds a
    tensor (and, under autograd, its gradient) to dt; the identity for dt None or float32.

    Passed as `rnd` to the layer and forecaster restatements below, it reproduces the
    precision a 16-bit implementation of them has at the boundaries where it stores 16-bit
    tensors (projection outputs, the prologue's XQ/XK/XV/XU/eta, the scan and mixing
    outputs, the post_norm rows, the wo output; the gradients of each), with exact
    arithmetic in between. The reference's own 16-bit training (autocast, main.py:87)
    rounds at the same kind of boundaries."""
    if dt is None or dt == torch.float32:
        return lambda x: x
    return lambda x: _Round.apply(x, dt)


def _ident(x):
    return x


# --------------------------------------------------------------------------- one step
def linear_step(W, b, ln_w, ln_b, XQ, XK, XV, eta):
    """One mini-batch of TTT-Linear in dual form (ops/ttt_linear.py:8-54).

    Shapes (leading dims broadcast): XQ/XK/XV [B,NH,CS,F], eta [B,NH,CS,CS],
    W [B,NH,F,F], b [B,NH,1,F], ln_w/ln_b [NH,1,F]. Returns (W', b', XQW).
    """
    Z1 = XK @ W + b
    target = XV - XK
    G = ln_fused_l2_bwd(Z1, target, ln_w, ln_b)
    Attn = XQ @ XK.transpose(-2, -1)
    b_bar = b - eta @ G
    Z1_bar = XQ @ W - (eta * Attn) @ G + b_bar
    last_eta = eta[:, :, -1, :, None]
    W_new = W - (last_eta * XK).transpose(-1, -2) @ G
    b_new = b - torch.sum(last_eta * G, dim=-2, keepdim=True)
    return W_new, b_new, XQ + ln_fwd(Z1_bar, ln_w, ln_b)


def mlp_step(W1, b1, W2, b2, ln_w, ln_b, XQ, XK, XV, eta):
    """One mini-batch of TTT-MLP in dual form (ops/ttt_mlp.py:9-67)."""
    Z1 = XK @ W1 + b1
    X2 = gelu_tanh(Z1)
    Z2 = X2 @ W2 + b2
    target = XV - XK
    G2 = ln_fused_l2_bwd(Z2, target, ln_w, ln_b)
    G1 = G2 @ W2.transpose(-2, -1) * gelu_bwd(Z1)
    Attn1 = XQ @ XK.transpose(-2, -1)
    b1_bar = b1 - eta @ G1
    Z1_bar = XQ @ W1 - (eta * Attn1) @ G1 + b1_bar
    X2_bar = gelu_tanh(Z1_bar)
    Attn2 = X2_bar @ X2.transpose(-2, -1)
    b2_bar = b2 - eta @ G2
    Z2_bar = X2_bar @ W2 - (eta * Attn2) @ G2 + b2_bar
    last_eta = eta[:, :, -1, :, None]
    W1_new = W1 - (last_eta * XK).transpose(-1, -2) @ G1
    b1_new = b1 - torch.sum(last_eta * G1, dim=-2, keepdim=True)
    W2_new = W2 - (last_eta * X2).transpose(-1, -2) @ G2
    b2_new = b2 - torch.sum(last_eta * G2, dim=-2, keepdim=True)
    return W1_new, b1_new, W2_new, b2_new, XQ + ln_fwd(Z2_bar, ln_w, ln_b)


# --------------------------------------------------------------------------- scans
def linear_scan(ln_w, ln_b, W1, b1, XQ, XV, XK, eta, checkpoint_group_size=1):
    """TTT-Linear over the whole sequence, kernel layout in and out.

    Inputs follow ``TritonLinear.apply`` (linear_triton.py:15-53): XQ/XV/XK
    [B,NH,NC,CS,F], eta [B,NH,NC,CS,CS], W1 [B,NH,F,F], b1 [B,NH,1,F], ln [NH,F].
    Returns a dict with XQW [B,NH,NC,CS,F], W_last, b_last and the checkpoints
    [B,NH,K,F,F] / [B,NH,K,1,F] (state at the start of each group,
    kernels/linear_forward.py:55-73).
    """
    B, NH, NC, CS, F = XQ.shape
    ckpt = max(int(checkpoint_group_size), 1)
    lw = ln_w.reshape(NH, 1, F)
    lb = ln_b.reshape(NH, 1, F)
    W, b = W1, b1
    outs, W_ck, b_ck = [], [], []
    for n in range(NC):
        if n % ckpt == 0:
            W_ck.append(W)
            b_ck.append(b)
        W, b, o = linear_step(W, b, lw, lb, XQ[:, :, n], XK[:, :, n], XV[:, :, n], eta[:, :, n])
        outs.append(o)
    return {
        "XQW": torch.stack(outs, dim=2),
        "W_last": W,
        "b_last": b,
        "W_ckpt": torch.stack(W_ck, dim=2),
        "b_ckpt": torch.stack(b_ck, dim=2),
    }


def mlp_scan(ln_w, ln_b, W1, b1, W2, b2, XQ, XV, XK, eta, checkpoint_group_size=1, memo_segment_size=1):
    """TTT-MLP over the whole sequence, kernel layout (mlp_triton.py:15-62).

    Returns XQW, final states, checkpoints (start of each group) and memo states
    (state after mini-batch i for i % memo_segment_size == 0,
    kernels/mlp_forward.py:193-226), each [B,NH,K|NS,...].
    """
    B, NH, NC, CS, F = XQ.shape
    ckpt = max(int(checkpoint_group_size), 1)
    memo = max(int(memo_segment_size), 1)
    lw = ln_w.reshape(NH, 1, F)
    lb = ln_b.reshape(NH, 1, F)
    st = (W1, b1, W2, b2)
    outs = []
    ck = [[], [], [], []]
    mm = [[], [], [], []]
    for n in range(NC):
        if n % ckpt == 0:
            for i in range(4):
                ck[i].append(st[i])
        *st, o = mlp_step(*st, lw, lb, XQ[:, :, n], XK[:, :, n], XV[:, :, n], eta[:, :, n])
        outs.append(o)
        if n % memo == 0:
            for i in range(4):
                mm[i].append(st[i])
    res = {"XQW": torch.stack(outs, dim=2)}
    for i, name in enumerate(("W1", "b1", "W2", "b2")):
        res[name + "_last"] = st[i]
        res[name + "_ckpt"] = torch.stack(ck[i], dim=2)
        res[name + "_memo"] = torch.stack(mm[i], dim=2)
    return res


def ttt_linear(XK, XQ, XV, eta, ttt_norm_weight, ttt_norm_bias, W1_init, b1_init, checkpoint_group_size):
    """``ops.ttt_linear`` signature and output layout [B,NC,CS,NH,F] (ops/ttt_linear.py:57-84)."""
    out = linear_scan(ttt_norm_weight, ttt_norm_bias, W1_init, b1_init, XQ, XV, XK, eta, checkpoint_group_size)
    return out["XQW"].permute(0, 2, 3, 1, 4)


def ttt_mlp(XK, XQ, XV, eta, ttt_norm_weight, ttt_norm_bias, W1_init, b1_init, W2_init, b2_init, checkpoint_group_size):
    """``ops.ttt_mlp`` signature and output layout [B,NC,CS,NH,F] (ops/ttt_mlp.py:70-99)."""
    out = mlp_scan(ttt_norm_weight, ttt_norm_bias, W1_init, b1_init, W2_init, b2_init, XQ, XV, XK, eta, checkpoint_group_size)
    return out["XQW"].permute(0, 2, 3, 1, 4)


def mlp_cached_readout(XQ_seg, W1, b1, W2, b2, ln_w, ln_b, eps=READOUT_EPS):
    """XQ + LN(gelu(XQ W1 + b1) W2 + b2) for a frozen state (kernels/mlp_cached_readout.py:88-101,143).

    XQ_seg [B,NH,NCseg,CS,F]; W1 [B,NH,F,FF]; b1 [B,NH,1,FF]; W2 [B,NH,FF,F];
    b2 [B,NH,1,F]; ln [NH,F]. The GELU is the kernel's tanh form
    (kernels/utils.py:9-14), i.e. the same function as F.gelu(approximate="tanh").
    """
    B, NH, NCs, CS, F = XQ_seg.shape
    Z1 = XQ_seg @ W1[:, :, None] + b1[:, :, None]
    X2 = gelu_tanh(Z1)
    Z2 = X2 @ W2[:, :, None] + b2[:, :, None]
    lw = ln_w.reshape(1, NH, 1, 1, F)
    lb = ln_b.reshape(1, NH, 1, 1, F)
    return XQ_seg + ln_fwd(Z2, lw, lb, eps=eps)


def memo_mix(XQW, XQ, XK, XU, W1_memo, b1_memo, W2_memo, b2_memo, ln_w, ln_b, memo_segment_size):
    """Memo-state mixing of the TTT-MLP layer's output (ttt_layer.py:503-559), all segments.

    XQW, XQ, XK, XU [B,NH,NC,CS,F]; memo states [B,NH,NS,...] from mlp_scan(..., memo_segment_size)
    (memo j = state after mini-batch j * memo_segment_size). Segment i covers mini-batches
    [i*M, min((i+1)*M, NC)). Its summary is the mean of its XK over mini-batches and tokens
    (ttt_layer.py:519); the summaries of earlier segments enter detached (:527, :558). For
    i >= 1 each token mixes, with softmax weights over sims_j = <XU, summary_j> (j = 0..i,
    :522-533), the online output (weight of j = i, :536) and the cached read-outs of memo
    states 0..i-1 (:540-554). Segment 0 passes through. Differentiable in XQW, XU and XK
    (through the current segment's summary); the cached read-outs carry no gradient (:542).
    """
    B, NH, NC, CS, F = XQW.shape
    M = int(memo_segment_size)
    NS = math.ceil(NC / M)
    out_segs = []
    cached = []
    for i in range(NS):
        s0, s1 = i * M, min((i + 1) * M, NC)
        XQ_seg = XQ[:, :, s0:s1]
        XU_seg = XU[:, :, s0:s1]
        XQW_seg = XQW[:, :, s0:s1]
        summary_cur = XK[:, :, s0:s1].mean(dim=(2, 3))
        if i == 0:
            cached.append(summary_cur.detach())
            out_segs.append(XQW_seg)
            continue
        sims = [(XU_seg * summ[:, :, None, None, :]).sum(dim=-1) for summ in cached]
        sims.append((XU_seg * summary_cur[:, :, None, None, :]).sum(dim=-1))
        gamma = torch.softmax(torch.stack(sims, dim=-1), dim=-1)
        seg = gamma[..., -1:] * XQW_seg
        for j in range(i):
            with torch.no_grad():
                delta = mlp_cached_readout(XQ_seg, W1_memo[:, :, j], b1_memo[:, :, j], W2_memo[:, :, j],
                                           b2_memo[:, :, j], ln_w, ln_b)
            seg = seg + gamma[..., j:j + 1] * delta
        out_segs.append(seg)
        cached.append(summary_cur.detach())
    return torch.cat(out_segs, dim=2)


def process_input(hidden, wq, bq, wk, bk, wv, bv, wu, bu, lr_w, lr_b, ln_w, ln_b, freqs_cos, freqs_sin,
                  mini_batch_size, base_lr, rnd=_ident):
    """The TTT layer's input prologue (ttt_layer.py:261-330 with no text prefix, no multi-scene
    interleave, no tensor parallelism): projections (:141-148), L2 normalisation of XQ, XK, XU
    (:276-278), rotary embedding of XQ, XK and XU (:284-295, utils.py:97-123), the LayerNorm
    reconstruction target XV <- LN(XV - XK) + XK with the unbiased std and eps 1e-8 added to it
    (:227-244), the kernel layout [B, NH, NC, CS, F] (:246-259) and the learning rate
    eta = 1/CS * base_lr * sigmoid(X w_h + b_h) / F repeated over rows (:150-163, :309).

    hidden [B, L, W]; w* [W, W], b* [W] (nn.Linear); lr_w [NH, 1, W], lr_b [NH, 1];
    ln_w, ln_b [NH, F]; freqs_cos / freqs_sin [L, F/2] (the real and imaginary parts of the
    layer's freqs_cis rows 0..L-1). Returns XQ, XK, XV, XU, eta. `rnd` (see rounding())
    rounds the projection weights and outputs and the five results.
    """
    B, L, W = hidden.shape
    NH = ln_w.shape[0]
    F = W // NH
    CS = int(mini_batch_size)
    NC = L // CS

    def heads(x):
        return x.reshape(B, L, NH, F)

    def rope(x):
        a, b = x[..., 0::2], x[..., 1::2]
        c = freqs_cos[:L].reshape(1, L, 1, F // 2)
        sn = freqs_sin[:L].reshape(1, L, 1, F // 2)
        return torch.stack((a * c - b * sn, a * sn + b * c), dim=-1).flatten(-2)

    hidden = rnd(hidden)

    def proj(w, b):
        return heads(rnd(hidden @ rnd(w).T + rnd(b)))

    XQ, XK, XV, XU = proj(wq, bq), proj(wk, bk), proj(wv, bv), proj(wu, bu)
    XQ = rope(Fn.normalize(XQ, p=2, dim=-1))
    XK = rope(Fn.normalize(XK, p=2, dim=-1))
    XU = rope(Fn.normalize(XU, p=2, dim=-1))
    Y = XV - XK
    Y = (Y - Y.mean(dim=-1, keepdim=True)) / (Y.std(dim=-1, keepdim=True) + 1e-8)
    XV = ln_w.reshape(1, 1, NH, F) * Y + ln_b.reshape(1, 1, NH, F) + XK

    def layout(x):
        return x.transpose(1, 2).reshape(B, NH, NC, CS, F)

    Xmb = hidden.reshape(B, NC, CS, W)
    lr = rnd(torch.einsum("bnkc,hdc->bhnkd", Xmb, rnd(lr_w)) + rnd(lr_b).reshape(1, -1, 1, 1, 1))
    lr = torch.sigmoid(lr).permute(0, 1, 2, 4, 3)  # [B, NH, NC, 1, CS]
    eta = (1.0 / CS) * (base_lr * lr / F).repeat(1, 1, 1, CS, 1)
    return {"XQ": rnd(layout(XQ)), "XK": rnd(layout(XK)), "XV": rnd(layout(XV)), "XU": rnd(layout(XU)),
            "eta": rnd(eta)}


PROLOGUE_PARAM_NAMES = ("hidden", "wq", "bq", "wk", "bk", "wv", "bv", "wu", "bu", "lr_w", "lr_b", "ln_w", "ln_b")


def process_input_grads(inp, douts, mini_batch_size, base_lr):
    """Autograd gradients of sum_k <out_k, douts[k]> w.r.t. every prologue input."""
    leaves = {k: inp[k].detach().clone().requires_grad_(True) for k in PROLOGUE_PARAM_NAMES}
    out = process_input(*(leaves[k] for k in PROLOGUE_PARAM_NAMES), inp["freqs_cos"], inp["freqs_sin"],
                        mini_batch_size, base_lr)
    loss = sum((out[k] * douts[k]).sum() for k in ("XQ", "XK", "XV", "XU", "eta"))
    loss.backward()
    return {k: leaves[k].grad for k in PROLOGUE_PARAM_NAMES}, {k: v.detach() for k, v in out.items()}


def post_norm_wo(XQW, pn_w, pn_b, wo_w, wo_b, eps=1e-6, rnd=_ident):
    """The layer's output epilogue: the scan output [B, NH, NC, CS, F] permuted to token order
    [B, L, NH * F] (ttt_layer.py:563-564), post_norm = LayerNorm over the width with eps 1e-6
    (:77, :349) and the wo projection (:350)."""
    B, NH, NC, CS, F = XQW.shape
    h = XQW.permute(0, 2, 3, 1, 4).reshape(B, NC * CS, NH * F)
    h = rnd(Fn.layer_norm(h, (NH * F,), pn_w, pn_b, eps))
    return rnd(h @ rnd(wo_w).T + rnd(wo_b))


EPILOGUE_PARAM_NAMES = ("XQW", "pn_w", "pn_b", "wo_w", "wo_b")


def post_norm_wo_grads(inp, dout, eps=1e-6):
    """Autograd gradients of <post_norm_wo(...), dout> w.r.t. every epilogue input."""
    leaves = {k: inp[k].detach().clone().requires_grad_(True) for k in EPILOGUE_PARAM_NAMES}
    out = post_norm_wo(*(leaves[k] for k in EPILOGUE_PARAM_NAMES), eps)
    (out * dout).sum().backward()
    return {k: leaves[k].grad for k in EPILOGUE_PARAM_NAMES}, out.detach()


def ttt_mlp_layer(P, pre, h, rope_cos, rope_sin, mini_batch_size, base_lr, checkpoint_group_size,
                  memo_segment_size, rnd=_ident):
    """One TTT-MLP layer's forward (TTTBase.forward, ttt_layer.py:337-357, with TTTMLP.ttt's
    kernel branch, :453-565): process_input, the scan, memo mixing and post_norm + wo.
    P holds the layer's parameters under the prefix `pre` (reference module names); `rnd`
    rounds the stage boundaries (rounding())."""
    def q(n):
        return P[pre + n]

    inp = process_input(h, q("wq.weight"), q("wq.bias"), q("wk.weight"), q("wk.bias"), q("wv.weight"),
                        q("wv.bias"), q("wu.weight"), q("wu.bias"), q("learnable_ttt_lr_weight"),
                        q("learnable_ttt_lr_bias"), q("ttt_norm_weight"), q("ttt_norm_bias"), rope_cos, rope_sin,
                        mini_batch_size, base_lr, rnd)
    B = h.shape[0]
    NC = inp["XV"].shape[2]
    ckpt = min(max(int(checkpoint_group_size), 1), NC)

    def tile(t):
        return t.unsqueeze(0).expand(B, *t.shape)

    r = mlp_scan(q("ttt_norm_weight"), q("ttt_norm_bias"), tile(q("W1")), tile(q("b1")), tile(q("W2")), tile(q("b2")),
                 inp["XQ"], inp["XV"], inp["XK"], inp["eta"], ckpt, memo_segment_size)
    XQW = rnd(memo_mix(rnd(r["XQW"]), inp["XQ"], inp["XK"], inp["XU"], r["W1_memo"].detach(), r["b1_memo"].detach(),
                       r["W2_memo"].detach(), r["b2_memo"].detach(), q("ttt_norm_weight"), q("ttt_norm_bias"),
                       memo_segment_size))
    return post_norm_wo(XQW, q("post_norm.weight"), q("post_norm.bias"), q("wo.weight"), q("wo.bias"), rnd=rnd)


def forecaster(P, x, layer_prefixes, rope_cos, rope_sin, pred_len, mini_batch_size, base_lr, checkpoint_group_size,
               memo_segment_size, rnd=_ident):
    """TTTForecaster.forward (forecast.py:94-99) with the TTT layers stacked: in_proj, each
    layer of `layer_prefixes` in turn, head on the last position. `rnd` rounds the input
    projection and every layer's stage boundaries (rounding()); the head runs unrounded."""
    h = rnd(rnd(x) @ rnd(P["in_proj.weight"]).T + rnd(P["in_proj.bias"]))
    for pre in layer_prefixes:
        h = ttt_mlp_layer(P, pre, h, rope_cos, rope_sin, mini_batch_size, base_lr, checkpoint_group_size,
                          memo_segment_size, rnd)
    out = h[:, -1] @ P["head.weight"].T + P["head.bias"]
    return out.view(x.shape[0], pred_len, -1)


def forecaster_grads(P, x, y, layer_prefixes, rope_cos, rope_sin, pred_len, mini_batch_size, base_lr,
                     checkpoint_group_size, memo_segment_size, rnd=_ident):
    """MSE loss (main.py:89) of the forecaster and its gradients w.r.t. every parameter."""
    leaves = {k: v.detach().clone().requires_grad_(True) for k, v in P.items()}
    out = forecaster(leaves, x, layer_prefixes, rope_cos, rope_sin, pred_len, mini_batch_size, base_lr,
                     checkpoint_group_size, memo_segment_size, rnd)
    loss = Fn.mse_loss(out, y)
    loss.backward()
    grads = {k: (v.grad if v.grad is not None else torch.zeros_like(v)) for k, v in leaves.items()}
    return grads, out.detach(), loss.detach()


MEMO_MIX_GRAD_NAMES = ("XQW", "XU", "XK")


def memo_mix_grads(inp, dO, memo_segment_size):
    """Autograd gradients of <memo_mix(...), dO> w.r.t. XQW, XU and XK."""
    leaves = {k: (inp[k].detach().clone().requires_grad_(True) if k in MEMO_MIX_GRAD_NAMES else inp[k])
              for k in inp}
    out = memo_mix(leaves["XQW"], leaves["XQ"], leaves["XK"], leaves["XU"], leaves["W1_memo"], leaves["b1_memo"],
                   leaves["W2_memo"], leaves["b2_memo"], leaves["ln_w"], leaves["ln_b"], memo_segment_size)
    out.backward(dO)
    return {k: leaves[k].grad for k in MEMO_MIX_GRAD_NAMES}, out.detach()


# --------------------------------------------------------------------------- gradients
LINEAR_GRAD_NAMES = ("ln_w", "ln_b", "W1", "b1", "XQ", "XV", "XK", "eta")
MLP_GRAD_NAMES = ("ln_w", "ln_b", "W1", "b1", "W2", "b2", "XQ", "XV", "XK", "eta")


def linear_grads(inp, dO):
    """Autograd gradients of <XQW, dO> w.r.t. every TritonLinear input (order of linear_triton.py:254-265)."""
    leaves = {k: inp[k].detach().clone().requires_grad_(True) for k in LINEAR_GRAD_NAMES}
    out = linear_scan(leaves["ln_w"], leaves["ln_b"], leaves["W1"], leaves["b1"], leaves["XQ"], leaves["XV"], leaves["XK"], leaves["eta"])
    out["XQW"].backward(dO)
    return {k: leaves[k].grad.detach() for k in LINEAR_GRAD_NAMES}, {k: v.detach() for k, v in out.items()}


def mlp_grads(inp, dO):
    """Autograd gradients of <XQW, dO> w.r.t. every TritonMLP input (order of mlp_triton.py:338-351)."""
    leaves = {k: inp[k].detach().clone().requires_grad_(True) for k in MLP_GRAD_NAMES}
    out = mlp_scan(
        leaves["ln_w"], leaves["ln_b"], leaves["W1"], leaves["b1"], leaves["W2"], leaves["b2"],
        leaves["XQ"], leaves["XV"], leaves["XK"], leaves["eta"],
    )
    out["XQW"].backward(dO)
    return {k: leaves[k].grad.detach() for k in MLP_GRAD_NAMES}, {k: v.detach() for k, v in out.items()}


def rel_l2(a, b):
    """Relative L2 error ||a - b|| / ||b|| in float64 (the parity metric of the build)."""
    a = torch.as_tensor(a).double()
    b = torch.as_tensor(b).double()
    den = torch.linalg.vector_norm(b)
    num = torch.linalg.vector_norm(a - b)
    if den == 0:
        return float(num)
    return float(num / den)


def num_checkpoints(NC, ckpt):
    return math.ceil(NC / max(int(ckpt), 1))
