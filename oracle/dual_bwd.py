"""Hand-derived backward of the dual-form TTT scan (the algorithm the CUDA backward kernels run).

TEST INFRASTRUCTURE ONLY (see ttt_oracle.py's header for the import rule). The
reference has no correct dual-form backward: its Triton backward is primal-form and
keeps only the last row of d(eta) (kernels/linear_backward.py:130-135). Its ``ops/``
path gets gradients from autograd through ops/ttt_linear.py:8-54 / ops/ttt_mlp.py:9-67.
This file writes that autograd out by hand, one mini-batch at a time, and
``tests/test_oracle.py`` checks it against ``ttt_oracle.linear_grads`` / ``mlp_grads``.

Structure (identical in the CUDA kernels):

* the forward stores the state at the start of every checkpoint group;
* for each group, last to first: re-run the group's inner forward from its checkpoint,
  keeping the per-mini-batch pre-activations Z (Linear) or Z1, Z2 (MLP); then walk the
  group backwards. The state entering mini-batch n is recovered from the state after it
  by undoing the rank-CS update, W_n = W_{n+1} + X^T diag(e) G_n, with G_n rebuilt
  from the stored Z (this is exact up to rounding and needs no per-step state copy);
* per mini-batch, the backward takes dO and the carried (dW, db) for the state after
  the step and returns the input gradients plus (dW, db) for the state before it.

Notation per mini-batch (C = CS rows, F features): e = eta[C-1, :] (the update row),
P = eta * (XQ XK^T + 1) so that Z_bar = XQ W + b - P G.
"""

from __future__ import annotations

import torch
import torch.nn.functional as Fn

from ttt_oracle import LN_EPS, gelu_bwd


def _stats(x, eps=LN_EPS):
    mu = x.mean(-1, keepdim=True)
    var = ((x - mu) ** 2).mean(-1, keepdim=True)
    std = torch.sqrt(var + eps)
    return (x - mu) / std, std


def ln_core_bwd(d, xh, std):
    """d/dx of a LayerNorm without affine, given d/d(x_hat)."""
    F = d.shape[-1]
    return (F * d - d.sum(-1, keepdim=True) - xh * (d * xh).sum(-1, keepdim=True)) / (F * std)


def ln_fused_fwd(Z, T, gamma, beta):
    """G = d/dZ 1/2||LN(Z) - T||^2 plus the pieces its backward reuses."""
    xh, std = _stats(Z)
    go = gamma * xh + beta - T  # grad_output
    gh = go * gamma  # grad_x_hat
    G = ln_core_bwd(gh, xh, std)
    return G, (xh, std, go, gh)


def ln_fused_bwd(dG, G, saved, gamma):
    """Backward of G = ln_fused_l2_bwd(Z, T) -> (dZ, dT, dgamma_rows, dbeta_rows)."""
    xh, std, go, gh = saved
    F = xh.shape[-1]
    dgh = ln_core_bwd(dG, xh, std)
    S2 = (gh * xh).sum(-1, keepdim=True)
    dGxh = (dG * xh).sum(-1, keepdim=True)
    dxh = -(dG * S2 + gh * dGxh) / (F * std) + dgh * gamma * gamma
    dstd = -(dG * G).sum(-1, keepdim=True) / std
    dZ = ln_core_bwd(dxh, xh, std) + dstd * xh / F
    dT = -dgh * gamma
    return dZ, dT, dgh * (go + gamma * xh), dgh * gamma


def gelu_grad(x):
    """Exact derivative of F.gelu(x, approximate='tanh') (what autograd applies)."""
    k0 = 0.7978845608028654
    k1 = 0.044715
    inner = k0 * (x + k1 * x * x * x)
    t = torch.tanh(inner)
    return 0.5 * (1 + t) + 0.5 * x * (1 - t * t) * k0 * (1 + 3 * k1 * x * x)


def gelu_bwd_grad(x):
    """Exact derivative of the reference's gelu_bwd expression (ops/ttt_utils.py:51-54)."""
    a = 0.79788456
    c = 0.1070322243
    k = 0.044715
    t = torch.tanh(a * x * (1 + k * x * x))
    dt = (1 - t * t) * (a + 3 * a * k * x * x)
    poly = a + c * x * x
    return 0.5 * (1 - t * t) * poly + 0.5 * x * (-2 * t * dt * poly + (1 - t * t) * 2 * c * x) + 0.5 * dt


def _colsum(x):
    return x.sum(-2, keepdim=True)


# --------------------------------------------------------------------------- Linear
def linear_step_bwd(W, b, gamma, beta, XQ, XK, XV, eta, dO, dWn, dbn):
    """Backward of one TTT-Linear mini-batch (ops/ttt_linear.py:8-54).

    W, b: state entering the step. dWn, dbn: gradient w.r.t. the state after it.
    Returns dict of per-step gradients; 'W', 'b' hold the gradient w.r.t. (W, b).
    """
    XKt = XK.transpose(-1, -2)
    e = eta[..., -1, :]  # [.., C]
    Z = XK @ W + b
    T = XV - XK
    G, saved = ln_fused_fwd(Z, T, gamma, beta)
    A = XQ @ XKt
    P = eta * (A + 1.0)
    Zb = XQ @ W + b - P @ G
    xb, sb = _stats(Zb)
    # readout LayerNorm
    dgamma = _colsum(dO * xb)
    dbeta = _colsum(dO)
    dZb = ln_core_bwd(dO * gamma, xb, sb)
    # Z_bar = XQ W + b - P G
    dXQ = dO + dZb @ W.transpose(-1, -2)
    dW = dWn + XQ.transpose(-1, -2) @ dZb
    db = dbn + _colsum(dZb)
    dP = -dZb @ G.transpose(-1, -2)
    dG = -P.transpose(-1, -2) @ dZb
    deta = dP * (A + 1.0)
    dA = dP * eta
    dXQ = dXQ + dA @ XK
    dXK = dA.transpose(-1, -2) @ XQ
    # W' = W - XK^T diag(e) G ; b' = b - e^T G
    XdW = XK @ dWn
    dG = dG - e[..., None] * (XdW + dbn)
    dXK = dXK - e[..., None] * (G @ dWn.transpose(-1, -2))
    de = -(XdW * G).sum(-1) - (G * dbn).sum(-1)
    deta = deta.clone()
    deta[..., -1, :] += de
    # G = ln_fused_l2_bwd(Z, T)
    dZ, dT, dg_rows, db_rows = ln_fused_bwd(dG, G, saved, gamma)
    dgamma = dgamma + _colsum(dg_rows)
    dbeta = dbeta + _colsum(db_rows)
    dXV = dT
    dXK = dXK - dT + dZ @ W.transpose(-1, -2)
    dW = dW + XKt @ dZ
    db = db + _colsum(dZ)
    return {"XQ": dXQ, "XK": dXK, "XV": dXV, "eta": deta, "W": dW, "b": db, "ln_w": dgamma, "ln_b": dbeta}


def linear_backward(inp, dO, ckpt):
    """Whole-sequence TTT-Linear backward with checkpoint-group recompute and state reversal.

    inp: dict in kernel layout (XQ, XK, XV, eta, W1, b1, ln_w, ln_b); dO [B,NH,NC,CS,F].
    Returns gradients in TritonLinear's order of names (ln_w, ln_b, W1, b1, XQ, XV, XK, eta).
    """
    XQ, XK, XV, eta = inp["XQ"], inp["XK"], inp["XV"], inp["eta"]
    B, NH, NC, C, F = XQ.shape
    gamma = inp["ln_w"].reshape(NH, 1, F)
    beta = inp["ln_b"].reshape(NH, 1, F)
    # forward: checkpoints at group starts
    W, b = inp["W1"], inp["b1"]
    ck = []
    for n in range(NC):
        if n % ckpt == 0:
            ck.append((W, b))
        Z = XK[:, :, n] @ W + b
        G, _ = ln_fused_fwd(Z, XV[:, :, n] - XK[:, :, n], gamma, beta)
        e = eta[:, :, n, -1, :, None]
        W = W - (e * XK[:, :, n]).transpose(-1, -2) @ G
        b = b - _colsum(e * G)
    out = {k: torch.zeros_like(inp[k]) for k in ("XQ", "XK", "XV", "eta")}
    dW = torch.zeros_like(inp["W1"])
    db = torch.zeros_like(inp["b1"])
    dgamma = torch.zeros(B, NH, 1, F, dtype=XQ.dtype)
    dbeta = torch.zeros(B, NH, 1, F, dtype=XQ.dtype)
    for k in range(len(ck) - 1, -1, -1):
        n0, n1 = k * ckpt, min((k + 1) * ckpt, NC)
        W, b = ck[k]
        Zs = []
        for n in range(n0, n1):  # group re-forward: keep Z only
            Z = XK[:, :, n] @ W + b
            Zs.append(Z)
            G, _ = ln_fused_fwd(Z, XV[:, :, n] - XK[:, :, n], gamma, beta)
            e = eta[:, :, n, -1, :, None]
            W = W - (e * XK[:, :, n]).transpose(-1, -2) @ G
            b = b - _colsum(e * G)
        for n in range(n1 - 1, n0 - 1, -1):  # reverse walk with state reversal
            G, _ = ln_fused_fwd(Zs[n - n0], XV[:, :, n] - XK[:, :, n], gamma, beta)
            e = eta[:, :, n, -1, :, None]
            W = W + (e * XK[:, :, n]).transpose(-1, -2) @ G
            b = b + _colsum(e * G)
            g = linear_step_bwd(W, b, gamma, beta, XQ[:, :, n], XK[:, :, n], XV[:, :, n], eta[:, :, n], dO[:, :, n], dW, db)
            for name in ("XQ", "XK", "XV", "eta"):
                out[name][:, :, n] = g[name]
            dW, db = g["W"], g["b"]
            dgamma = dgamma + g["ln_w"]
            dbeta = dbeta + g["ln_b"]
    return {
        "ln_w": dgamma.sum(0).reshape(NH, F),
        "ln_b": dbeta.sum(0).reshape(NH, F),
        "W1": dW,
        "b1": db,
        **out,
    }


# --------------------------------------------------------------------------- MLP
def mlp_step_bwd(W1, b1, W2, b2, gamma, beta, XQ, XK, XV, eta, dO, dW1n, db1n, dW2n, db2n):
    """Backward of one TTT-MLP mini-batch (ops/ttt_mlp.py:9-67)."""
    XKt = XK.transpose(-1, -2)
    e = eta[..., -1, :]
    Z1 = XK @ W1 + b1
    X2 = Fn.gelu(Z1, approximate="tanh")
    Z2 = X2 @ W2 + b2
    T = XV - XK
    G2, saved = ln_fused_fwd(Z2, T, gamma, beta)
    H = G2 @ W2.transpose(-1, -2)
    gp = gelu_bwd(Z1)
    G1 = H * gp
    A1 = XQ @ XKt
    P1 = eta * (A1 + 1.0)
    Z1b = XQ @ W1 + b1 - P1 @ G1
    X2b = Fn.gelu(Z1b, approximate="tanh")
    A2 = X2b @ X2.transpose(-1, -2)
    P2 = eta * (A2 + 1.0)
    Z2b = X2b @ W2 + b2 - P2 @ G2
    xb, sb = _stats(Z2b)
    # readout LayerNorm
    dgamma = _colsum(dO * xb)
    dbeta = _colsum(dO)
    dZ2b = ln_core_bwd(dO * gamma, xb, sb)
    # Z2_bar = X2_bar W2 + b2 - P2 G2
    dX2b = dZ2b @ W2.transpose(-1, -2)
    dW2 = dW2n + X2b.transpose(-1, -2) @ dZ2b
    db2 = db2n + _colsum(dZ2b)
    dP2 = -dZ2b @ G2.transpose(-1, -2)
    dG2 = -P2.transpose(-1, -2) @ dZ2b
    deta = dP2 * (A2 + 1.0)
    dA2 = dP2 * eta
    dX2b = dX2b + dA2 @ X2
    dX2 = dA2.transpose(-1, -2) @ X2b
    # X2_bar = gelu(Z1_bar)
    dZ1b = dX2b * gelu_grad(Z1b)
    # Z1_bar = XQ W1 + b1 - P1 G1
    dXQ = dO + dZ1b @ W1.transpose(-1, -2)
    dW1 = dW1n + XQ.transpose(-1, -2) @ dZ1b
    db1 = db1n + _colsum(dZ1b)
    dP1 = -dZ1b @ G1.transpose(-1, -2)
    dG1 = -P1.transpose(-1, -2) @ dZ1b
    deta = deta + dP1 * (A1 + 1.0)
    dA1 = dP1 * eta
    dXQ = dXQ + dA1 @ XK
    dXK = dA1.transpose(-1, -2) @ XQ
    # updates
    XdW1 = XK @ dW1n
    dG1 = dG1 - e[..., None] * (XdW1 + db1n)
    dXK = dXK - e[..., None] * (G1 @ dW1n.transpose(-1, -2))
    de = -(XdW1 * G1).sum(-1) - (G1 * db1n).sum(-1)
    XdW2 = X2 @ dW2n
    dG2 = dG2 - e[..., None] * (XdW2 + db2n)
    dX2 = dX2 - e[..., None] * (G2 @ dW2n.transpose(-1, -2))
    de = de - (XdW2 * G2).sum(-1) - (G2 * db2n).sum(-1)
    deta = deta.clone()
    deta[..., -1, :] += de
    # G1 = (G2 W2^T) * gelu_bwd(Z1)
    dH = dG1 * gp
    dZ1 = dG1 * H * gelu_bwd_grad(Z1)
    dG2 = dG2 + dH @ W2
    dW2 = dW2 + dH.transpose(-1, -2) @ G2
    # G2 = ln_fused_l2_bwd(Z2, T)
    dZ2, dT, dg_rows, db_rows = ln_fused_bwd(dG2, G2, saved, gamma)
    dgamma = dgamma + _colsum(dg_rows)
    dbeta = dbeta + _colsum(db_rows)
    # Z2 = X2 W2 + b2 ; X2 = gelu(Z1) ; Z1 = XK W1 + b1 ; T = XV - XK
    dX2 = dX2 + dZ2 @ W2.transpose(-1, -2)
    dW2 = dW2 + X2.transpose(-1, -2) @ dZ2
    db2 = db2 + _colsum(dZ2)
    dZ1 = dZ1 + dX2 * gelu_grad(Z1)
    dXK = dXK + dZ1 @ W1.transpose(-1, -2) - dT
    dW1 = dW1 + XKt @ dZ1
    db1 = db1 + _colsum(dZ1)
    return {
        "XQ": dXQ, "XK": dXK, "XV": dT, "eta": deta,
        "W1": dW1, "b1": db1, "W2": dW2, "b2": db2, "ln_w": dgamma, "ln_b": dbeta,
    }


def _mlp_inner(W1, b1, W2, b2, gamma, beta, XK, XV, eta_n):
    Z1 = XK @ W1 + b1
    X2 = Fn.gelu(Z1, approximate="tanh")
    Z2 = X2 @ W2 + b2
    G2, _ = ln_fused_fwd(Z2, XV - XK, gamma, beta)
    G1 = (G2 @ W2.transpose(-1, -2)) * gelu_bwd(Z1)
    return Z1, X2, Z2, G1, G2


def mlp_backward(inp, dO, ckpt):
    """Whole-sequence TTT-MLP backward (same structure as ``linear_backward``).

    State reversal for the MLP: W2_n = W2_{n+1} + X2^T diag(e) G2 (X2, G2 from the stored
    Z1, Z2), then G1 = (G2 W2_n^T) * gelu_bwd(Z1) and W1_n = W1_{n+1} + XK^T diag(e) G1.
    """
    XQ, XK, XV, eta = inp["XQ"], inp["XK"], inp["XV"], inp["eta"]
    B, NH, NC, C, F = XQ.shape
    gamma = inp["ln_w"].reshape(NH, 1, F)
    beta = inp["ln_b"].reshape(NH, 1, F)
    st = [inp["W1"], inp["b1"], inp["W2"], inp["b2"]]
    ck = []
    for n in range(NC):
        if n % ckpt == 0:
            ck.append(list(st))
        Z1, X2, Z2, G1, G2 = _mlp_inner(*st, gamma, beta, XK[:, :, n], XV[:, :, n], eta[:, :, n])
        e = eta[:, :, n, -1, :, None]
        st = [st[0] - (e * XK[:, :, n]).transpose(-1, -2) @ G1, st[1] - _colsum(e * G1),
              st[2] - (e * X2).transpose(-1, -2) @ G2, st[3] - _colsum(e * G2)]
    out = {k: torch.zeros_like(inp[k]) for k in ("XQ", "XK", "XV", "eta")}
    dst = [torch.zeros_like(inp[k]) for k in ("W1", "b1", "W2", "b2")]
    dgamma = torch.zeros(B, NH, 1, F, dtype=XQ.dtype)
    dbeta = torch.zeros(B, NH, 1, F, dtype=XQ.dtype)
    for k in range(len(ck) - 1, -1, -1):
        n0, n1 = k * ckpt, min((k + 1) * ckpt, NC)
        st = list(ck[k])
        Zs = []
        for n in range(n0, n1):
            Z1, X2, Z2, G1, G2 = _mlp_inner(*st, gamma, beta, XK[:, :, n], XV[:, :, n], eta[:, :, n])
            Zs.append((Z1, Z2))
            e = eta[:, :, n, -1, :, None]
            st = [st[0] - (e * XK[:, :, n]).transpose(-1, -2) @ G1, st[1] - _colsum(e * G1),
                  st[2] - (e * X2).transpose(-1, -2) @ G2, st[3] - _colsum(e * G2)]
        for n in range(n1 - 1, n0 - 1, -1):
            Z1, Z2 = Zs[n - n0]
            e = eta[:, :, n, -1, :, None]
            X2 = Fn.gelu(Z1, approximate="tanh")
            G2, _ = ln_fused_fwd(Z2, XV[:, :, n] - XK[:, :, n], gamma, beta)
            st[2] = st[2] + (e * X2).transpose(-1, -2) @ G2
            st[3] = st[3] + _colsum(e * G2)
            G1 = (G2 @ st[2].transpose(-1, -2)) * gelu_bwd(Z1)
            st[0] = st[0] + (e * XK[:, :, n]).transpose(-1, -2) @ G1
            st[1] = st[1] + _colsum(e * G1)
            g = mlp_step_bwd(*st, gamma, beta, XQ[:, :, n], XK[:, :, n], XV[:, :, n], eta[:, :, n], dO[:, :, n], *dst)
            for name in ("XQ", "XK", "XV", "eta"):
                out[name][:, :, n] = g[name]
            dst = [g["W1"], g["b1"], g["W2"], g["b2"]]
            dgamma = dgamma + g["ln_w"]
            dbeta = dbeta + g["ln_b"]
    return {
        "ln_w": dgamma.sum(0).reshape(NH, F),
        "ln_b": dbeta.sum(0).reshape(NH, F),
        "W1": dst[0], "b1": dst[1], "W2": dst[2], "b2": dst[3],
        **out,
    }
