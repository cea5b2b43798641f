"""Functional host side of the B200 TTT scan: shape checks, allocation, C-ABI launches.

Every function here allocates its outputs with ``torch.empty`` on the inputs' device
(as the reference wrappers do, linear_triton.py:81-88, mlp_triton.py:102-119), makes the
inputs contiguous, and enqueues one kernel on the current CUDA stream. None of them
synchronises the device.
"""

from __future__ import annotations

import functools
import math

import torch

from _lib import check, dtype_code, lib, ptr, require_cuda, stream_of


def _c(t):
    return t.contiguous()


def _on_tensor_device(fn):
    """Run an entry point with its first tensor argument's device current: the library
    launches on the current device and resolves the per-device error word, scratch address
    and tensor maps there, while the stream comes from the tensors' device."""

    @functools.wraps(fn)
    def wrapper(*args, **kwargs):
        for a in args:
            if isinstance(a, torch.Tensor):
                if a.is_cuda and a.device.index != torch.cuda.current_device():
                    with torch.cuda.device(a.device):
                        return fn(*args, **kwargs)
                break
        return fn(*args, **kwargs)

    return wrapper


def _check_acts(XQ, XV, XK, eta):
    if XQ.dim() != 5:
        raise ValueError(f"XQ must be [B, NH, NC, CS, F], got shape {tuple(XQ.shape)}")
    B, NH, NC, CS, F = XQ.shape
    for name, t in (("XV", XV), ("XK", XK)):
        if tuple(t.shape) != (B, NH, NC, CS, F):
            raise ValueError(f"{name} must have XQ's shape {tuple(XQ.shape)}, got {tuple(t.shape)}")
    if tuple(eta.shape) != (B, NH, NC, CS, CS):
        raise ValueError(f"eta must be [B, NH, NC, CS, CS] = {(B, NH, NC, CS, CS)}, got {tuple(eta.shape)}")
    return B, NH, NC, CS, F


def _check_ln(ln_w, ln_b, NH, F):
    for name, t in (("ttt_norm_weight", ln_w), ("ttt_norm_bias", ln_b)):
        if t.numel() != NH * F:
            raise ValueError(f"{name} must have NH * F = {NH * F} elements, got shape {tuple(t.shape)}")
    if ln_w.dtype != ln_b.dtype:
        ln_b = ln_b.to(ln_w.dtype)
    return _c(ln_w), _c(ln_b)


def _state(t, shape, name):
    if tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name} must be {tuple(shape)}, got {tuple(t.shape)}")
    return t.to(torch.float32).contiguous()


# --------------------------------------------------------------------------- Linear
@_on_tensor_device
def linear_forward(ln_w, ln_b, W1, b1, XQ, XV, XK, eta, checkpoint_group_size, for_backward=True):
    """TTT-Linear scan forward. Returns (XQW in XQ's dtype, W_last, b_last, W_ckpt, b_ckpt, Z).

    With ``for_backward`` the group-start checkpoints and the fp32 pre-activations Z of
    every mini-batch are kept for ``linear_backward``; without it (inference) neither is
    written and both come back as None."""
    require_cuda(ln_w, ln_b, W1, b1, XQ, XV, XK, eta)
    B, NH, NC, CS, F = _check_acts(XQ, XV, XK, eta)
    ckpt = int(checkpoint_group_size)
    if ckpt <= 0:
        raise ValueError(f"checkpoint_group_size must be positive, got {ckpt}")
    K = math.ceil(NC / ckpt)
    ln_w, ln_b = _check_ln(ln_w, ln_b, NH, F)
    W1 = _state(W1, (B, NH, F, F), "W1_init")
    b1 = _state(b1, (B, NH, 1, F), "b1_init")
    XQ, XV, XK, eta = _c(XQ), _c(XV), _c(XK), _c(eta)
    dev = XQ.device
    XQW = torch.empty(B, NH, NC, CS, F, device=dev, dtype=XQ.dtype)
    W_last = torch.empty(B, NH, F, F, device=dev, dtype=torch.float32)
    b_last = torch.empty(B, NH, 1, F, device=dev, dtype=torch.float32)
    W_ckpt = b_ckpt = Z = None
    if for_backward:
        W_ckpt = torch.empty(B, NH, K, F, F, device=dev, dtype=torch.float32)
        b_ckpt = torch.empty(B, NH, K, 1, F, device=dev, dtype=torch.float32)
        Z = torch.empty(B, NH, NC, CS, F, device=dev, dtype=torch.float32)
    rc = lib.ttt_linear_fwd(
        B, NH, NC, CS, F, ckpt,
        ptr(ln_w), ptr(ln_b), dtype_code(ln_w),
        ptr(W1), ptr(b1),
        ptr(XQ), dtype_code(XQ), ptr(XV), dtype_code(XV), ptr(XK), dtype_code(XK),
        ptr(eta), dtype_code(eta),
        ptr(XQW), dtype_code(XQW),
        ptr(W_last), ptr(b_last), ptr(W_ckpt), ptr(b_ckpt), ptr(Z),
        stream_of(XQ),
    )
    check(rc, "ttt_linear_fwd")
    return XQW, W_last, b_last, W_ckpt, b_ckpt, Z


@_on_tensor_device
def linear_backward(ln_w, ln_b, W_ckpt, b_ckpt, XQ, XV, XK, eta, dXQW, checkpoint_group_size, grad_dtype=None,
                    Z=None, W_last=None, b_last=None):
    """TTT-Linear scan backward. Returns (d_ln_w [B,NH,F] per-(b,h) partials, d_ln_b,
    dW1, db1 (fp32), dXQ, dXV, dXK, d_eta (grad_dtype, default XQ's dtype)).

    ``Z``, ``W_last``, ``b_last`` (from ``linear_forward``) enable the single reverse walk;
    without them each checkpoint group is re-run forward."""
    require_cuda(ln_w, ln_b, W_ckpt, b_ckpt, XQ, XV, XK, eta, dXQW)
    if Z is not None:
        require_cuda(Z, W_last, b_last)
        Z, W_last, b_last = _c(Z), _c(W_last), _c(b_last)
    B, NH, NC, CS, F = _check_acts(XQ, XV, XK, eta)
    ckpt = int(checkpoint_group_size)
    ln_w, ln_b = _check_ln(ln_w, ln_b, NH, F)
    if tuple(dXQW.shape) != tuple(XQ.shape):
        raise ValueError(f"upstream gradient must have XQ's shape {tuple(XQ.shape)}, got {tuple(dXQW.shape)}")
    XQ, XV, XK, eta, dXQW = _c(XQ), _c(XV), _c(XK), _c(eta), _c(dXQW)
    W_ckpt, b_ckpt = _c(W_ckpt), _c(b_ckpt)
    gdt = grad_dtype or XQ.dtype
    dev = XQ.device
    d_ln_w = torch.empty(B, NH, F, device=dev, dtype=torch.float32)
    d_ln_b = torch.empty(B, NH, F, device=dev, dtype=torch.float32)
    dW1 = torch.empty(B, NH, F, F, device=dev, dtype=torch.float32)
    db1 = torch.empty(B, NH, 1, F, device=dev, dtype=torch.float32)
    dXQ = torch.empty(B, NH, NC, CS, F, device=dev, dtype=gdt)
    dXV = torch.empty_like(dXQ)
    dXK = torch.empty_like(dXQ)
    deta = torch.empty(B, NH, NC, CS, CS, device=dev, dtype=gdt)
    nbytes = lib.ttt_linear_bwd_scratch_bytes(B, NH, NC, CS, F, ckpt)
    scratch = torch.empty(max(nbytes, 1), device=dev, dtype=torch.uint8)
    rc = lib.ttt_linear_bwd(
        B, NH, NC, CS, F, ckpt,
        ptr(ln_w), ptr(ln_b), dtype_code(ln_w),
        ptr(W_ckpt), ptr(b_ckpt),
        ptr(XQ), dtype_code(XQ), ptr(XV), dtype_code(XV), ptr(XK), dtype_code(XK),
        ptr(eta), dtype_code(eta),
        ptr(dXQW), dtype_code(dXQW),
        ptr(Z), ptr(W_last), ptr(b_last),
        ptr(d_ln_w), ptr(d_ln_b), ptr(dW1), ptr(db1),
        ptr(dXQ), ptr(dXV), ptr(dXK), ptr(deta), dtype_code(dXQ),
        ptr(scratch), nbytes, stream_of(XQ),
    )
    check(rc, "ttt_linear_bwd")
    return d_ln_w, d_ln_b, dW1, db1, dXQ, dXV, dXK, deta


# --------------------------------------------------------------------------- MLP
@_on_tensor_device
def mlp_forward(ln_w, ln_b, W1, b1, W2, b2, XQ, XV, XK, eta, checkpoint_group_size, memo_segment_size=None,
                for_backward=True):
    """TTT-MLP scan forward. Returns (XQW, (W1,b1,W2,b2)_last, (…)_ckpt or None, (…)_memo or None,
    (Z1, Z2, Z1bar, Z2bar) or None).

    With ``for_backward`` the checkpoints and the fp32 pre-activations of every mini-batch
    are kept for ``mlp_backward``; without it (inference) neither is written."""
    require_cuda(ln_w, ln_b, W1, b1, W2, b2, XQ, XV, XK, eta)
    B, NH, NC, CS, F = _check_acts(XQ, XV, XK, eta)
    FF = W1.shape[-1]
    ckpt = int(checkpoint_group_size)
    if ckpt <= 0:
        raise ValueError(f"checkpoint_group_size must be positive, got {ckpt}")
    K = math.ceil(NC / ckpt)
    ln_w, ln_b = _check_ln(ln_w, ln_b, NH, F)
    W1 = _state(W1, (B, NH, F, FF), "W1_init")
    b1 = _state(b1, (B, NH, 1, FF), "b1_init")
    W2 = _state(W2, (B, NH, FF, F), "W2_init")
    b2 = _state(b2, (B, NH, 1, F), "b2_init")
    XQ, XV, XK, eta = _c(XQ), _c(XV), _c(XK), _c(eta)
    dev = XQ.device
    f32 = dict(device=dev, dtype=torch.float32)
    XQW = torch.empty(B, NH, NC, CS, F, device=dev, dtype=XQ.dtype)
    last = (torch.empty(B, NH, F, FF, **f32), torch.empty(B, NH, 1, FF, **f32),
            torch.empty(B, NH, FF, F, **f32), torch.empty(B, NH, 1, F, **f32))
    ck = None
    if for_backward:
        ck = (torch.empty(B, NH, K, F, FF, **f32), torch.empty(B, NH, K, 1, FF, **f32),
              torch.empty(B, NH, K, FF, F, **f32), torch.empty(B, NH, K, 1, F, **f32))
    cp = ck if ck is not None else (None, None, None, None)
    memo = None
    memo_seg = 1
    if memo_segment_size is not None:
        memo_seg = int(memo_segment_size)
        if memo_seg <= 0:
            raise ValueError(f"memo_segment_size must be positive, got {memo_seg}")
        NS = math.ceil(NC / memo_seg)
        memo = (torch.empty(B, NH, NS, F, FF, **f32), torch.empty(B, NH, NS, 1, FF, **f32),
                torch.empty(B, NH, NS, FF, F, **f32), torch.empty(B, NH, NS, 1, F, **f32))
    mp = memo if memo is not None else (None, None, None, None)
    zs = None
    if for_backward:
        zs = (torch.empty(B, NH, NC, CS, FF, **f32), torch.empty(B, NH, NC, CS, F, **f32),
              torch.empty(B, NH, NC, CS, FF, **f32), torch.empty(B, NH, NC, CS, F, **f32))
    zp = zs if zs is not None else (None, None, None, None)
    rc = lib.ttt_mlp_fwd(
        B, NH, NC, CS, F, FF, ckpt, memo_seg,
        ptr(ln_w), ptr(ln_b), dtype_code(ln_w),
        ptr(W1), ptr(b1), ptr(W2), ptr(b2),
        ptr(XQ), dtype_code(XQ), ptr(XV), dtype_code(XV), ptr(XK), dtype_code(XK),
        ptr(eta), dtype_code(eta),
        ptr(XQW), dtype_code(XQW),
        *[ptr(t) for t in last], *[ptr(t) for t in cp], *[ptr(t) for t in mp], *[ptr(t) for t in zp],
        stream_of(XQ),
    )
    check(rc, "ttt_mlp_fwd")
    return XQW, last, ck, memo, zs


@_on_tensor_device
def mlp_backward(ln_w, ln_b, ckpts, XQ, XV, XK, eta, dXQW, checkpoint_group_size, grad_dtype=None,
                 saved=None, W1_last=None, W2_last=None):
    """TTT-MLP scan backward. ckpts = (W1, b1, W2, b2) checkpoints from mlp_forward.
    Returns (d_ln_w, d_ln_b [B,NH,F] partials, dW1, db1, dW2, db2, dXQ, dXV, dXK, d_eta).

    ``saved`` = (Z1, Z2, Z1bar, Z2bar) from ``mlp_forward`` with the final W1 and W2
    enable the single reverse walk; without them each checkpoint group is re-run forward."""
    W1c, b1c, W2c, b2c = (_c(t) for t in ckpts)
    require_cuda(ln_w, ln_b, W1c, b1c, W2c, b2c, XQ, XV, XK, eta, dXQW)
    sp = (None,) * 6
    if saved is not None:
        if W1_last is None or W2_last is None:
            raise ValueError("saved pre-activations need W1_last and W2_last")
        sp = tuple(_c(t) for t in (*saved, W1_last, W2_last))
        require_cuda(*sp)
    B, NH, NC, CS, F = _check_acts(XQ, XV, XK, eta)
    FF = W1c.shape[-1]
    ckpt = int(checkpoint_group_size)
    ln_w, ln_b = _check_ln(ln_w, ln_b, NH, F)
    if tuple(dXQW.shape) != tuple(XQ.shape):
        raise ValueError(f"upstream gradient must have XQ's shape {tuple(XQ.shape)}, got {tuple(dXQW.shape)}")
    XQ, XV, XK, eta, dXQW = _c(XQ), _c(XV), _c(XK), _c(eta), _c(dXQW)
    gdt = grad_dtype or XQ.dtype
    dev = XQ.device
    f32 = dict(device=dev, dtype=torch.float32)
    d_ln_w = torch.empty(B, NH, F, **f32)
    d_ln_b = torch.empty(B, NH, F, **f32)
    dW1 = torch.empty(B, NH, F, FF, **f32)
    db1 = torch.empty(B, NH, 1, FF, **f32)
    dW2 = torch.empty(B, NH, FF, F, **f32)
    db2 = torch.empty(B, NH, 1, F, **f32)
    dXQ = torch.empty(B, NH, NC, CS, F, device=dev, dtype=gdt)
    dXV = torch.empty_like(dXQ)
    dXK = torch.empty_like(dXQ)
    deta = torch.empty(B, NH, NC, CS, CS, device=dev, dtype=gdt)
    nbytes = lib.ttt_mlp_bwd_scratch_bytes(B, NH, NC, CS, F, FF, ckpt)
    scratch = torch.empty(max(nbytes, 1), device=dev, dtype=torch.uint8)
    rc = lib.ttt_mlp_bwd(
        B, NH, NC, CS, F, FF, ckpt,
        ptr(ln_w), ptr(ln_b), dtype_code(ln_w),
        ptr(W1c), ptr(b1c), ptr(W2c), ptr(b2c),
        ptr(XQ), dtype_code(XQ), ptr(XV), dtype_code(XV), ptr(XK), dtype_code(XK),
        ptr(eta), dtype_code(eta),
        ptr(dXQW), dtype_code(dXQW),
        *[ptr(t) for t in sp],
        ptr(d_ln_w), ptr(d_ln_b), ptr(dW1), ptr(db1), ptr(dW2), ptr(db2),
        ptr(dXQ), ptr(dXV), ptr(dXK), ptr(deta), dtype_code(dXQ),
        ptr(scratch), nbytes, stream_of(XQ),
    )
    check(rc, "ttt_mlp_bwd")
    return d_ln_w, d_ln_b, dW1, db1, dW2, db2, dXQ, dXV, dXK, deta


def _lead_strides(t, inner_numel, name):
    """Batch / head element strides of a [B, NH, ...] fp32 state whose trailing block is contiguous."""
    if t.dtype != torch.float32:
        t = t.to(torch.float32)
    inner = t.shape[2:]
    expect = 1
    for d in range(t.dim() - 1, 1, -1):
        if t.stride(d) != expect:
            t = t.contiguous()
            break
        expect *= t.shape[d]
    if math.prod(inner) != inner_numel:
        raise ValueError(f"{name} has shape {tuple(t.shape)}, trailing block must hold {inner_numel} elements")
    return t, t.stride(0), t.stride(1)


@_on_tensor_device
def mlp_cached_readout(XQ_seg, W1, b1, W2, b2, ln_w, ln_b):
    """XQ_seg + LN(gelu(XQ_seg W1 + b1) W2 + b2) in fp32 (LN eps 1e-6)."""
    require_cuda(XQ_seg, W1, b1, W2, b2, ln_w, ln_b)
    if XQ_seg.dim() != 5:
        raise ValueError(f"XQ_seg must be [B, NH, NCseg, CS, F], got {tuple(XQ_seg.shape)}")
    B, NH, NCs, CS, F = XQ_seg.shape
    FF = W1.shape[-1]
    for name, t, lead in (("W1", W1, (B, NH)), ("b1", b1, (B, NH)), ("W2", W2, (B, NH)), ("b2", b2, (B, NH))):
        if tuple(t.shape[:2]) != lead:
            raise ValueError(f"{name} must start with [B, NH] = {lead}, got {tuple(t.shape)}")
    W1, W1_sb, W1_sh = _lead_strides(W1, F * FF, "W1")
    b1, b1_sb, b1_sh = _lead_strides(b1, FF, "b1")
    W2, W2_sb, W2_sh = _lead_strides(W2, FF * F, "W2")
    b2, b2_sb, b2_sh = _lead_strides(b2, F, "b2")
    ln_w, ln_b = _check_ln(ln_w, ln_b, NH, F)
    XQ_seg = _c(XQ_seg)
    out = torch.empty(B, NH, NCs, CS, F, device=XQ_seg.device, dtype=torch.float32)
    rc = lib.ttt_mlp_cached_readout(
        B, NH, NCs, CS, F, FF, ptr(XQ_seg), dtype_code(XQ_seg),
        ptr(W1), W1_sb, W1_sh, ptr(b1), b1_sb, b1_sh,
        ptr(W2), W2_sb, W2_sh, ptr(b2), b2_sb, b2_sh,
        ptr(ln_w), ptr(ln_b), dtype_code(ln_w), ptr(out), stream_of(XQ_seg),
    )
    check(rc, "ttt_mlp_cached_readout")
    return out


# --------------------------------------------------------------------------- memo mixing
def _memo_args(XQW, XQ, XK, XU, W1_memo, b1_memo, W2_memo, b2_memo, ln_w, ln_b, memo_segment_size):
    require_cuda(XQW, XQ, XK, XU, W1_memo, b1_memo, W2_memo, b2_memo, ln_w, ln_b)
    if XQW.dim() != 5:
        raise ValueError(f"XQW must be [B, NH, NC, CS, F], got {tuple(XQW.shape)}")
    B, NH, NC, CS, F = XQW.shape
    for name, t in (("XQ", XQ), ("XK", XK), ("XU", XU)):
        if tuple(t.shape) != tuple(XQW.shape):
            raise ValueError(f"{name} must have XQW's shape {tuple(XQW.shape)}, got {tuple(t.shape)}")
        if t.dtype != XQW.dtype:
            raise ValueError(f"{name} must have XQW's dtype {XQW.dtype}, got {t.dtype}")
    M = int(memo_segment_size)
    if M <= 0:
        raise ValueError(f"memo_segment_size must be positive, got {M}")
    NS = math.ceil(NC / M)
    FF = W1_memo.shape[-1]
    mem = (_state(W1_memo, (B, NH, NS, F, FF), "W1_memo"), _state(b1_memo, (B, NH, NS, 1, FF), "b1_memo"),
           _state(W2_memo, (B, NH, NS, FF, F), "W2_memo"), _state(b2_memo, (B, NH, NS, 1, F), "b2_memo"))
    ln_w, ln_b = _check_ln(ln_w, ln_b, NH, F)
    return (B, NH, NC, CS, F, FF, M), (_c(XQW), _c(XQ), _c(XK), _c(XU)), mem, ln_w, ln_b


@_on_tensor_device
def memo_mix_forward(XQW, XQ, XK, XU, W1_memo, b1_memo, W2_memo, b2_memo, ln_w, ln_b, memo_segment_size,
                     return_scratch=False):
    """Memo-state mixing of the TTT-MLP output (ttt_layer.py:503-559) as one launch sequence.
    Returns the mixed output in XQW's dtype and layout [B, NH, NC, CS, F]; with
    return_scratch, also the scratch holding the prepared memo operands and summaries, which
    memo_mix_backward reuses."""
    dims, acts, mem, ln_w, ln_b = _memo_args(XQW, XQ, XK, XU, W1_memo, b1_memo, W2_memo, b2_memo, ln_w, ln_b,
                                             memo_segment_size)
    B, NH, NC, CS, F, FF, M = dims
    XQW, XQ, XK, XU = acts
    out = torch.empty_like(XQW)
    nbytes = lib.ttt_memo_mix_scratch_bytes(B, NH, NC, M, FF)
    scratch = torch.empty(max(nbytes, 1), device=XQW.device, dtype=torch.uint8)
    rc = lib.ttt_memo_mix_fwd(
        B, NH, NC, CS, F, FF, M, ptr(XQW), ptr(XQ), ptr(XK), ptr(XU), dtype_code(XQW),
        *[ptr(t) for t in mem], ptr(ln_w), ptr(ln_b), dtype_code(ln_w),
        ptr(out), ptr(scratch), nbytes, stream_of(XQW),
    )
    check(rc, "ttt_memo_mix_fwd")
    return (out, scratch) if return_scratch else out


@_on_tensor_device
def memo_mix_backward(XQW, XQ, XK, XU, W1_memo, b1_memo, W2_memo, b2_memo, ln_w, ln_b, memo_segment_size, dOut,
                      scratch=None):
    """Gradients of the memo mixing: (dXQW, dXU, dXK), dXK being the part through the
    segment summaries (the cached read-outs carry none, ttt_layer.py:542). `scratch` may be
    the one memo_mix_forward returned for the same inputs (its prepared operands are reused)."""
    dims, acts, mem, ln_w, ln_b = _memo_args(XQW, XQ, XK, XU, W1_memo, b1_memo, W2_memo, b2_memo, ln_w, ln_b,
                                             memo_segment_size)
    B, NH, NC, CS, F, FF, M = dims
    XQW, XQ, XK, XU = acts
    if tuple(dOut.shape) != tuple(XQW.shape):
        raise ValueError(f"upstream gradient must have XQW's shape {tuple(XQW.shape)}, got {tuple(dOut.shape)}")
    dOut = _c(dOut.to(XQW.dtype))
    dXQW, dXU, dXK = torch.empty_like(XQW), torch.empty_like(XQW), torch.empty_like(XQW)
    nbytes = lib.ttt_memo_mix_scratch_bytes(B, NH, NC, M, FF)
    prepped = scratch is not None
    if prepped:
        if scratch.numel() < nbytes or scratch.device != XQW.device:
            raise ValueError("the forward's scratch does not match these inputs")
    else:
        scratch = torch.empty(max(nbytes, 1), device=XQW.device, dtype=torch.uint8)
    rc = lib.ttt_memo_mix_bwd(
        B, NH, NC, CS, F, FF, M, ptr(XQW), ptr(XQ), ptr(XK), ptr(XU), dtype_code(XQW),
        *[ptr(t) for t in mem], ptr(ln_w), ptr(ln_b), dtype_code(ln_w),
        ptr(dOut), ptr(dXQW), ptr(dXU), ptr(dXK), ptr(scratch), nbytes, int(prepped), stream_of(XQW),
    )
    check(rc, "ttt_memo_mix_bwd")
    return dXQW, dXU, dXK


# --------------------------------------------------------------------------- input prologue
def prologue_ld(NH, F):
    """Row stride of the projection matrix: q | k | v | u (NH * F each) | NH gates, padded to 8."""
    n = 4 * NH * F + NH
    return (n + 7) // 8 * 8


def _prologue_args(P, B, L, NH, F, CS, ln_w, ln_b, rope_cos, rope_sin):
    require_cuda(P, ln_w, ln_b, rope_cos, rope_sin)
    ld = prologue_ld(NH, F)
    if P.dim() != 2 or tuple(P.shape) != (B * L, ld) or not P.is_contiguous():
        raise ValueError(f"projections must be a contiguous [B * L, {ld}] matrix, got {tuple(P.shape)}")
    if L % CS:
        raise ValueError(f"sequence length {L} must be a multiple of mini_batch_size {CS}")
    ln_w, ln_b = _check_ln(ln_w.to(torch.float32), ln_b.to(torch.float32), NH, F)
    for name, t in (("rope_cos", rope_cos), ("rope_sin", rope_sin)):
        if tuple(t.shape) != (L, F // 2) or t.dtype != torch.float32:
            raise ValueError(f"{name} must be float32 [{L}, {F // 2}], got {t.dtype} {tuple(t.shape)}")
    return ld, ln_w, ln_b, _c(rope_cos), _c(rope_sin)


@_on_tensor_device
def prologue_forward(P, B, L, NH, F, CS, ln_w, ln_b, rope_cos, rope_sin, eta_scale):
    """Element-wise prologue over the projection matrix P ([B * L, prologue_ld], biases
    included). Returns XQ, XK, XV, XU [B, NH, NC, CS, F] and eta [B, NH, NC, CS, CS] in P's dtype."""
    ld, ln_w, ln_b, rope_cos, rope_sin = _prologue_args(P, B, L, NH, F, CS, ln_w, ln_b, rope_cos, rope_sin)
    NC = L // CS
    outs = [torch.empty(B, NH, NC, CS, F, device=P.device, dtype=P.dtype) for _ in range(4)]
    eta = torch.empty(B, NH, NC, CS, CS, device=P.device, dtype=P.dtype)
    rc = lib.ttt_prologue_fwd(
        B, L, NH, F, CS, ptr(P), dtype_code(P), ld, ptr(ln_w), ptr(ln_b), ptr(rope_cos), ptr(rope_sin),
        float(eta_scale), *(ptr(o) for o in outs), ptr(eta), stream_of(P),
    )
    check(rc, "ttt_prologue_fwd")
    return (*outs, eta)


@_on_tensor_device
def prologue_backward(P, B, L, NH, F, CS, ln_w, ln_b, rope_cos, rope_sin, eta_scale, dXQ, dXK, dXV, dXU, deta):
    """Gradient of the element-wise prologue: returns dP ([B * L, prologue_ld], P's dtype;
    padding columns zero), d ln_w, d ln_b ([NH, F] fp32) and the column sums of dP (the
    projection bias gradient, [prologue_ld] fp32). Gradients may be None."""
    ld, ln_w, ln_b, rope_cos, rope_sin = _prologue_args(P, B, L, NH, F, CS, ln_w, ln_b, rope_cos, rope_sin)
    NC = L // CS
    grads = []
    for name, g, shape in (("dXQ", dXQ, (B, NH, NC, CS, F)), ("dXK", dXK, (B, NH, NC, CS, F)),
                           ("dXV", dXV, (B, NH, NC, CS, F)), ("dXU", dXU, (B, NH, NC, CS, F)),
                           ("d_eta", deta, (B, NH, NC, CS, CS))):
        if g is not None:
            if tuple(g.shape) != shape:
                raise ValueError(f"{name} must be {shape}, got {tuple(g.shape)}")
            g = _c(g.to(P.dtype))
        grads.append(g)
    dP = torch.empty_like(P)
    dln_w = torch.zeros(NH, F, device=P.device, dtype=torch.float32)
    dln_b = torch.zeros(NH, F, device=P.device, dtype=torch.float32)
    dbias = torch.zeros(ld, device=P.device, dtype=torch.float32)
    rc = lib.ttt_prologue_bwd(
        B, L, NH, F, CS, ptr(P), dtype_code(P), ld, ptr(ln_w), ptr(ln_b), ptr(rope_cos), ptr(rope_sin),
        float(eta_scale), *(ptr(g) for g in grads), ptr(dP), ptr(dln_w), ptr(dln_b), ptr(dbias), stream_of(P),
    )
    check(rc, "ttt_prologue_bwd")
    return dP, dln_w, dln_b, dbias


# --------------------------------------------------------------------------- output epilogue
def _post_norm_args(XQW, ln_w, ln_b):
    require_cuda(XQW, ln_w, ln_b)
    if XQW.dim() != 5:
        raise ValueError(f"XQW must be [B, NH, NC, CS, F], got shape {tuple(XQW.shape)}")
    B, NH, NC, CS, F = XQW.shape
    W = NH * F
    if ln_w.numel() != W or ln_b.numel() != W:
        raise ValueError(f"post_norm weight and bias must have NH * F = {W} elements")
    return B, NH, NC * CS, F, _c(XQW), _c(ln_w.to(torch.float32)), _c(ln_b.to(torch.float32))


@_on_tensor_device
def post_norm_forward(XQW, ln_w, ln_b, eps):
    """LayerNorm over the width of the scan output, read in its kernel layout: returns the
    normalised rows [B * L, NH * F] in XQW's dtype (token order)."""
    B, NH, L, F, XQW, ln_w, ln_b = _post_norm_args(XQW, ln_w, ln_b)
    Y = torch.empty(B * L, NH * F, device=XQW.device, dtype=XQW.dtype)
    rc = lib.ttt_post_norm_fwd(B, NH, L, F, ptr(XQW), dtype_code(XQW), ptr(ln_w), ptr(ln_b), float(eps), ptr(Y),
                               stream_of(XQW))
    check(rc, "ttt_post_norm_fwd")
    return Y


@_on_tensor_device
def post_norm_backward(XQW, ln_w, ln_b, eps, dY, dOut=None):
    """Gradient of post_norm_forward: returns d XQW (kernel layout, XQW's dtype), the
    LayerNorm weight / bias gradients ([NH * F] fp32) and, when dOut (the gradient of the wo
    output, [B * L, NH * F]) is given, its column sums (the wo bias gradient, fp32) else None."""
    B, NH, L, F, XQW, ln_w, ln_b = _post_norm_args(XQW, ln_w, ln_b)
    for name, t in (("dY", dY), ("dOut", dOut)):
        if t is not None and tuple(t.shape) != (B * L, NH * F):
            raise ValueError(f"{name} must be [{B * L}, {NH * F}], got {tuple(t.shape)}")
    dY = _c(dY.to(XQW.dtype))
    dOut = _c(dOut.to(XQW.dtype)) if dOut is not None else None
    dX = torch.empty_like(XQW)
    dln_w = torch.zeros(NH * F, device=XQW.device, dtype=torch.float32)
    dln_b = torch.zeros(NH * F, device=XQW.device, dtype=torch.float32)
    dbias = torch.zeros(NH * F, device=XQW.device, dtype=torch.float32) if dOut is not None else None
    rc = lib.ttt_post_norm_bwd(B, NH, L, F, ptr(XQW), dtype_code(XQW), ptr(ln_w), ptr(ln_b), float(eps), ptr(dY),
                               ptr(dX), ptr(dln_w), ptr(dln_b), ptr(dOut), ptr(dbias), stream_of(XQW))
    check(rc, "ttt_post_norm_bwd")
    return dX, dln_w, dln_b, dbias
