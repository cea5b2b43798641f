"""Input prologue of the TTT layer on the sm_100a kernels: TTTBase.process_input
(ttt_layer.py:261-330) for the forecaster's case (no text prefix, no multi-scene
interleave, no tensor parallelism).

The reference runs four nn.Linear projections, a learning-rate einsum and about twenty
element-wise PyTorch ops, each a pass over HBM. Here the five projections are ONE library
GEMM into a [B * L, 4 * W + NH] matrix (biases fused), and a single kernel does the L2
normalisation, rotary embedding, LayerNorm reconstruction target, re-layout into the scan's
[B, NH, NC, CS, F] tiles and the eta gate; its backward is one kernel plus the two GEMMs
of the projection gradient. A maintainer switches the layer over with

    inputs = prologue.process_input(self, hidden_states, freqs_cis, seq_metadata)

in TTTBase.forward (ttt_layer.py:345) instead of ``self.process_input(...)``; the returned
dict has the reference's keys and shapes (XQ, XK, XV, XU, eta).
"""

from __future__ import annotations

import torch

import _core


def rope_tables(freqs_cis, L, F):
    """fp32 (cos, sin) [L, F/2] from the layer's complex freqs_cis ([>= L, F/2]) or a
    (cos, sin) pair of real tensors."""
    if isinstance(freqs_cis, (tuple, list)):
        cos, sin = freqs_cis
    else:
        if not torch.is_complex(freqs_cis):
            raise TypeError("freqs_cis must be a complex tensor [>= L, head_dim / 2] or a (cos, sin) pair")
        cos, sin = freqs_cis.real, freqs_cis.imag
    if cos.dim() != 2 or cos.shape[0] < L or cos.shape[1] != F // 2 or sin.shape != cos.shape:
        raise ValueError(f"rotary tables must be [>= {L}, {F // 2}], got {tuple(cos.shape)} and {tuple(sin.shape)}")
    return cos[:L].to(torch.float32).contiguous(), sin[:L].to(torch.float32).contiguous()


_ZERO_ROWS = {}


def _zero_rows(shape, like):
    """A cached all-zero padding block (never written: torch.cat only reads it)."""
    key = (tuple(shape), like.dtype, like.device)
    if key not in _ZERO_ROWS:
        _ZERO_ROWS[key] = torch.zeros(shape, dtype=like.dtype, device=like.device)
    return _ZERO_ROWS[key]


def concat_projections(wq, bq, wk, bk, wv, bv, wu, bu, lr_w, lr_b):
    """The five projections as one [prologue_ld, W] weight and bias (zero padding rows)."""
    NH = lr_w.shape[0]
    Wout, Win = wq.shape
    if Wout % NH:
        raise ValueError(f"projection width {Wout} is not a multiple of num_heads {NH}")
    F = Wout // NH
    ld = _core.prologue_ld(NH, F)
    pad = ld - (4 * Wout + NH)
    ws = [wq, wk, wv, wu, lr_w.reshape(NH, Win)]
    bs = [bq, bk, bv, bu, lr_b.reshape(NH)]
    if pad:
        ws.append(_zero_rows((pad, Win), wq))
        bs.append(_zero_rows((pad,), bq))
    return torch.cat(ws, 0), torch.cat(bs, 0), NH, F


class Prologue(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden, Wcat, bcat, ln_w, ln_b, rope_cos, rope_sin, NH, F, CS, base_lr):
        B, L, Win = hidden.shape
        h2 = hidden.reshape(B * L, Win)
        if not h2.is_contiguous():
            h2 = h2.contiguous()
        P = torch.addmm(bcat, h2, Wcat.t())  # one library GEMM: [B * L, prologue_ld]
        scale = float(base_lr) / (F * CS)
        outs = _core.prologue_forward(P, B, L, NH, F, CS, ln_w, ln_b, rope_cos, rope_sin, scale)
        ctx.set_materialize_grads(False)  # unused outputs (XU in TTT-Linear) reach the kernel as NULL
        ctx.dims = (B, L, Win, NH, F, CS, scale)
        ctx.ln_dtypes = (ln_w.dtype, ln_b.dtype)
        ctx.save_for_backward(h2, Wcat, P, ln_w, ln_b, rope_cos, rope_sin)
        return outs

    @staticmethod
    def backward(ctx, dXQ, dXK, dXV, dXU, deta):
        h2, Wcat, P, ln_w, ln_b, rope_cos, rope_sin = ctx.saved_tensors
        B, L, Win, NH, F, CS, scale = ctx.dims
        dP, dln_w, dln_b, dbias = _core.prologue_backward(P, B, L, NH, F, CS, ln_w, ln_b, rope_cos, rope_sin,
                                                          scale, dXQ, dXK, dXV, dXU, deta)
        # dP's padding columns are zero and so are Wcat's padding rows: both GEMMs run over the
        # full 8-aligned width.
        dhidden = torch.mm(dP, Wcat).reshape(B, L, Win)
        dWcat = torch.mm(dP.t(), h2)
        return (dhidden, dWcat, dbias.to(Wcat.dtype), dln_w.to(ctx.ln_dtypes[0]), dln_b.to(ctx.ln_dtypes[1]),
                None, None, None, None, None, None)


def ttt_prologue(hidden_states, wq, bq, wk, bk, wv, bv, wu, bu, learnable_ttt_lr_weight, learnable_ttt_lr_bias,
                 ttt_norm_weight, ttt_norm_bias, freqs_cis, mini_batch_size, ttt_base_lr):
    """process_input as a function of the layer's parameters. hidden_states [B, L, W];
    w* [NH * F, W] and b* [NH * F] (nn.Linear); learnable_ttt_lr_weight [NH, 1, W],
    learnable_ttt_lr_bias [NH, 1]; ttt_norm_weight / ttt_norm_bias [NH, F]; freqs_cis complex
    [>= L, F / 2] or (cos, sin). Returns {XQ, XK, XV, XU: [B, NH, NC, CS, F], eta:
    [B, NH, NC, CS, CS]} in hidden_states' dtype, differentiable w.r.t. every tensor input
    except freqs_cis."""
    if hidden_states.dim() != 3:
        raise ValueError(f"hidden_states must be [B, L, W], got {tuple(hidden_states.shape)}")
    B, L, Win = hidden_states.shape
    CS = int(mini_batch_size)
    if CS < 1 or L % CS:
        raise ValueError(f"sequence length {L} must be a multiple of mini_batch_size {CS}")
    if wq.shape[1] != Win:
        raise ValueError(f"projection input width {wq.shape[1]} != hidden width {Win}")
    dt = hidden_states.dtype
    Wcat, bcat, NH, F = concat_projections(wq, bq, wk, bk, wv, bv, wu, bu, learnable_ttt_lr_weight,
                                           learnable_ttt_lr_bias)
    rope_cos, rope_sin = rope_tables(freqs_cis, L, F)
    rope_cos, rope_sin = rope_cos.to(hidden_states.device), rope_sin.to(hidden_states.device)
    XQ, XK, XV, XU, eta = Prologue.apply(hidden_states, Wcat.to(dt), bcat.to(dt), ttt_norm_weight, ttt_norm_bias,
                                         rope_cos, rope_sin, NH, F, CS, float(ttt_base_lr))
    return {"XQ": XQ, "XK": XK, "XV": XV, "XU": XU, "eta": eta}


def process_input(layer, hidden_states, freqs_cis, seq_metadata=None):
    """Drop-in for ``layer.process_input(hidden_states, freqs_cis, seq_metadata)`` of a
    TTTBase layer (ttt_layer.py:261-330): reads the layer's wq/wk/wv/wu, learning-rate gate,
    TTT LayerNorm parameters, mini_batch_size and ttt_base_lr."""
    if seq_metadata is not None and getattr(seq_metadata, "is_multiscene", False):
        raise NotImplementedError("multi-scene interleaving is not part of the fused prologue")
    if getattr(layer, "tp_mesh", None) is not None:
        raise NotImplementedError("tensor-parallel inputs are not part of the fused prologue")
    return ttt_prologue(hidden_states, layer.wq.weight, layer.wq.bias, layer.wk.weight, layer.wk.bias,
                        layer.wv.weight, layer.wv.bias, layer.wu.weight, layer.wu.bias,
                        layer.learnable_ttt_lr_weight, layer.learnable_ttt_lr_bias, layer.ttt_norm_weight,
                        layer.ttt_norm_bias, freqs_cis, layer.mini_batch_size, layer.ttt_base_lr)
