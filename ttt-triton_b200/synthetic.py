"""Seeded synthetic inputs with the shapes and value distributions of the benchmark configs.

The reference benchmarks nothing itself; its configs (batch, heads, sequence, head dim,
mini-batch 16, inner width) are reproduced here with seeded data:

* XQ, XK, XV ~ N(0, 1) / 8 in kernel layout [B, NH, NC, CS, F];
* W ~ N(0, 0.02^2), biases 0, LayerNorm gamma = 1, beta = 0 (ttt_layer.py:81-89, 363-364);
* eta in the full [B, NH, NC, CS, CS] layout the kernels take:
  - ``"causal"``: eta[b,h,n,i,j] = s[b,h,n,j] / (i + 1) for j <= i, else 0, with
    s = sigmoid(N(0, 1)) / 64 (a per-token learning rate with a 1/(i+1) factor; the
    [j <= i] mask makes the reference's unmasked eta * Attn equal the causal dual form);
  - ``"equal"``: eta[b,h,n,i,j] = s[b,h,n,j] / CS for every row i, which is what the
    forecaster's layer feeds (ttt_layer.py:151-163, 309).
* upstream gradient dZ ~ N(0, 1) for backward.

Generation runs on ``device`` with a generator seeded there, so the large configs are
created directly in HBM.
"""

from __future__ import annotations

import torch


def _randn(shape, gen, device, dtype=torch.float32):
    return torch.randn(shape, generator=gen, device=device, dtype=dtype)


def make_eta(s, mode="causal"):
    """Build the [.., CS, CS] eta matrix from per-token rates s [.., CS]."""
    CS = s.shape[-1]
    idx = torch.arange(CS, device=s.device)
    if mode == "causal":
        scale = 1.0 / (idx.to(s.dtype) + 1.0)  # row i -> 1/(i+1)
        mask = (idx[None, :] <= idx[:, None]).to(s.dtype)  # [i, j] = j <= i
        return s[..., None, :] * (scale[:, None] * mask)
    if mode == "equal":
        return (s[..., None, :] / CS).expand(*s.shape[:-1], CS, CS).contiguous()
    raise ValueError(f"unknown eta mode {mode!r}")


def make_linear_inputs(B, NH, NC, CS=16, F=64, dtype=torch.float32, device="cpu", seed=0, eta_mode="causal"):
    """Inputs of ``TritonLinear.apply`` (linear_triton.py:15-53) as a dict."""
    g = torch.Generator(device=device).manual_seed(seed)
    d = {}
    d["XQ"] = (_randn((B, NH, NC, CS, F), g, device) / 8).to(dtype)
    d["XK"] = (_randn((B, NH, NC, CS, F), g, device) / 8).to(dtype)
    d["XV"] = (_randn((B, NH, NC, CS, F), g, device) / 8).to(dtype)
    s = torch.sigmoid(_randn((B, NH, NC, CS), g, device)) / 64
    d["eta"] = make_eta(s, eta_mode).to(dtype)
    W = _randn((NH, F, F), g, device) * 0.02
    d["W1"] = W[None].expand(B, NH, F, F).contiguous()
    d["b1"] = torch.zeros(B, NH, 1, F, device=device)
    d["ln_w"] = torch.ones(NH, F, device=device)
    d["ln_b"] = torch.zeros(NH, F, device=device)
    return d


def make_mlp_inputs(B, NH, NC, CS=16, F=64, FF=256, dtype=torch.float32, device="cpu", seed=0, eta_mode="causal"):
    """Inputs of ``TritonMLP.apply`` (mlp_triton.py:15-62) as a dict."""
    g = torch.Generator(device=device).manual_seed(seed)
    d = {}
    d["XQ"] = (_randn((B, NH, NC, CS, F), g, device) / 8).to(dtype)
    d["XK"] = (_randn((B, NH, NC, CS, F), g, device) / 8).to(dtype)
    d["XV"] = (_randn((B, NH, NC, CS, F), g, device) / 8).to(dtype)
    s = torch.sigmoid(_randn((B, NH, NC, CS), g, device)) / 64
    d["eta"] = make_eta(s, eta_mode).to(dtype)
    W1 = _randn((NH, F, FF), g, device) * 0.02
    W2 = _randn((NH, FF, F), g, device) * 0.02
    d["W1"] = W1[None].expand(B, NH, F, FF).contiguous()
    d["b1"] = torch.zeros(B, NH, 1, FF, device=device)
    d["W2"] = W2[None].expand(B, NH, FF, F).contiguous()
    d["b2"] = torch.zeros(B, NH, 1, F, device=device)
    d["ln_w"] = torch.ones(NH, F, device=device)
    d["ln_b"] = torch.zeros(NH, F, device=device)
    return d


def make_memo_inputs(B, NH, NC, CS=16, F=64, FF=256, memo_segment_size=16, dtype=torch.float32, device="cpu",
                     seed=0):
    """Inputs of the memo-state mixing at a layer's shapes: the scan output XQW, XQ, XK and the
    mixing query XU ~ N(0,1)/8 (XQW ~ N(0,1)), memo states near the MLP's initialisation
    (W ~ N(0, 0.02^2), biases ~ N(0, 0.01^2)) as TritonMLP returns them [B,NH,NS,...], LN
    weight 1 and bias 0."""
    g = torch.Generator(device=device).manual_seed(seed)
    NS = -(-NC // memo_segment_size)
    d = {
        "XQW": _randn((B, NH, NC, CS, F), g, device).to(dtype),
        "XQ": (_randn((B, NH, NC, CS, F), g, device) / 8).to(dtype),
        "XK": (_randn((B, NH, NC, CS, F), g, device) / 8).to(dtype),
        "XU": (_randn((B, NH, NC, CS, F), g, device) / 8).to(dtype),
        "W1_memo": _randn((B, NH, NS, F, FF), g, device) * 0.02,
        "b1_memo": _randn((B, NH, NS, 1, FF), g, device) * 0.01,
        "W2_memo": _randn((B, NH, NS, FF, F), g, device) * 0.02,
        "b2_memo": _randn((B, NH, NS, 1, F), g, device) * 0.01,
        "ln_w": torch.ones(NH, F, device=device),
        "ln_b": torch.zeros(NH, F, device=device),
    }
    return d


def rope_cos_sin(L, F, theta=10000.0, device="cpu"):
    """fp32 [L, F/2] cosine and sine tables of the standard 1-D rotary frequencies
    theta^(-2i/F) at positions 0..L-1 (the kernels take any table; the reference layer builds
    its freqs_cis with a 3-D variant, utils.py)."""
    inv = theta ** (-torch.arange(0, F, 2, dtype=torch.float64, device=device) / F)
    ang = torch.arange(L, dtype=torch.float64, device=device)[:, None] * inv[None, :]
    return torch.cos(ang).float(), torch.sin(ang).float()


def make_prologue_inputs(B, L, W, NH, device="cpu", seed=0):
    """A TTT layer's input prologue at the given shapes (fp32): hidden ~ N(0, 1) [B, L, W];
    projection weights ~ N(0, 0.02^2) and gate weight ~ N(0, 0.02^2) as init_weights
    (ttt_layer.py:81-89), biases ~ N(0, 0.02^2), gate bias ~ N(0, 0.5^2) and LayerNorm
    gamma ~ 1 + N(0, 0.1^2), beta ~ N(0, 0.1^2) so every gradient is exercised; rotary
    tables from rope_cos_sin."""
    g = torch.Generator(device=device).manual_seed(seed)
    F = W // NH
    d = {"hidden": _randn((B, L, W), g, device)}
    for k in ("q", "k", "v", "u"):
        d["w" + k] = _randn((W, W), g, device) * 0.02
        d["b" + k] = _randn((W,), g, device) * 0.02
    d["lr_w"] = _randn((NH, 1, W), g, device) * 0.02
    d["lr_b"] = _randn((NH, 1), g, device) * 0.5
    d["ln_w"] = 1.0 + 0.1 * _randn((NH, F), g, device)
    d["ln_b"] = 0.1 * _randn((NH, F), g, device)
    d["freqs_cos"], d["freqs_sin"] = rope_cos_sin(L, F, device=device)
    return d


def make_forecast_series(n_steps=17420, channels=7, seed=0):
    """The config-4 stand-in for an hourly multichannel series (ETTh1's length): channel k is
    a_k sin(2 pi t / 24 + phi_k) + b_k sin(2 pi t / 168 + psi_k) + 0.001 c_k t + AR(1) noise
    (rho 0.9, innovation sigma 0.3), a, b ~ U(0.5, 2), c ~ U(-1, 1), phases ~ U(0, 2 pi),
    z-normalised per channel. Returns fp32 [n_steps, channels] on the CPU."""
    import numpy as np

    rng = np.random.default_rng(seed)
    t = np.arange(n_steps, dtype=np.float64)[:, None]
    a, b = rng.uniform(0.5, 2.0, channels), rng.uniform(0.5, 2.0, channels)
    c = rng.uniform(-1.0, 1.0, channels)
    phi, psi = rng.uniform(0, 2 * np.pi, channels), rng.uniform(0, 2 * np.pi, channels)
    z = rng.standard_normal((n_steps, channels)) * 0.3
    noise = np.empty_like(z)
    noise[0] = z[0]
    for i in range(1, n_steps):
        noise[i] = 0.9 * noise[i - 1] + z[i]
    x = a * np.sin(2 * np.pi * t / 24 + phi) + b * np.sin(2 * np.pi * t / 168 + psi) + 0.001 * c * t + noise
    x = (x - x.mean(0)) / x.std(0)
    return torch.from_numpy(x.astype(np.float32))


def forecast_windows(series, lookback, horizon, batch, gen):
    """`batch` random windows of a [T, C] series: inputs [batch, lookback, C] and targets the
    following `horizon` steps [batch, horizon, C] (a torch.Generator picks the starts)."""
    T = series.shape[0]
    starts = torch.randint(0, T - lookback - horizon + 1, (batch,), generator=gen)
    idx = starts[:, None] + torch.arange(lookback + horizon)[None, :]
    w = series[idx]
    return w[:, :lookback].contiguous(), w[:, lookback:].contiguous()


def make_upstream(shape, device="cpu", seed=1, dtype=torch.float32):
    """dZ ~ N(0, 1) with the output's shape."""
    g = torch.Generator(device=device).manual_seed(seed)
    return _randn(shape, g, device).to(dtype)


def perturb_params(d, device="cpu", seed=2, scale=0.1):
    """Non-trivial LN params and biases so their gradients are exercised (tests only)."""
    g = torch.Generator(device=device).manual_seed(seed)
    out = dict(d)
    out["ln_w"] = d["ln_w"] + scale * _randn(d["ln_w"].shape, g, device)
    out["ln_b"] = d["ln_b"] + scale * _randn(d["ln_b"].shape, g, device)
    for k in ("b1", "b2"):
        if k in d:
            out[k] = d[k] + 0.02 * _randn(d[k].shape, g, device)
    return out
