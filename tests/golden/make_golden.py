"""Generate the golden vectors that pin the CPU oracle to the reference.

Run in a container that has the reference checkout (read-only is fine):

    python tests/golden/make_golden.py /path/to/ttt-triton

It imports the reference's own ``ops`` package (the PyTorch dual-form path,
ops/ttt_linear.py:57-84, ops/ttt_mlp.py:70-99) with TorchDynamo disabled (CPU Inductor
cannot build here) and ``forecast`` imported first (ttt_layer <-> forecast import
cycle), runs it in float64 on seeded float32-representable inputs, and takes gradients
with torch autograd exactly as the reference's training path does. The cached-readout
golden runs the reference's Triton kernel (kernels/mlp_cached_readout.py:7-109) under
the Triton CPU interpreter at B = NH = 1, the only slice its offsets address correctly; the
memo-mixing golden runs the reference's own mixing loop of TTTMLP.ttt with that kernel, the
prologue golden the layer's own process_input, the epilogue golden its forward tail and the
forecaster golden the reference's TTTForecaster with its scan launch on the ops path.

Outputs ``tests/golden/*.npz`` (float32 storage). The GPU box never runs this script.
"""

from __future__ import annotations

import os
import sys

os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")
os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "ttt-triton_b200"))
import synthetic  # noqa: E402  (seeded generators shared with the tests and bench)

sys.path.remove(os.path.join(REPO, "ttt-triton_b200"))
for name in [m for m in sys.modules if m == "ops" or m.startswith("ops.") or m == "kernels" or m.startswith("kernels.")]:
    del sys.modules[name]


def _np(t):
    return t.detach().to(torch.float32).cpu().numpy()


def _grads(fn, leaves, dO):
    leaves = {k: v.detach().clone().requires_grad_(True) for k, v in leaves.items()}
    out = fn(**leaves)
    out.backward(dO)
    return out.detach(), {k: v.grad.detach() for k, v in leaves.items()}


def linear_case(ref_ops, B, NH, NC, F, ckpt, eta_mode, seed, with_grads=True, perturb=True):
    d = synthetic.make_linear_inputs(B, NH, NC, 16, F, seed=seed, eta_mode=eta_mode)
    if perturb:
        d = synthetic.perturb_params(d, seed=seed + 7)
    d = {k: v.float() for k, v in d.items()}  # float32-representable inputs
    d64 = {k: v.double() for k, v in d.items()}

    def fn(XQ, XK, XV, eta, ln_w, ln_b, W1, b1):
        return ref_ops.ttt_linear(XK, XQ, XV, eta, ln_w, ln_b, W1, b1, ckpt)  # [B,NC,CS,NH,F]

    leaves = {k: d64[k] for k in ("XQ", "XK", "XV", "eta", "ln_w", "ln_b", "W1", "b1")}
    res = {("in_" + k): _np(v) for k, v in d.items()}
    res["ckpt"] = np.array(ckpt)
    if with_grads:
        dO = synthetic.make_upstream((B, NC, 16, NH, F), seed=seed + 1).double()
        out, grads = _grads(fn, leaves, dO)
        res["dO"] = _np(dO)
        res.update({("grad_" + k): _np(v) for k, v in grads.items()})
    else:
        with torch.no_grad():
            out = fn(**leaves)
    res["out"] = _np(out)
    return res


def mlp_case(ref_ops, B, NH, NC, F, FF, ckpt, eta_mode, seed, with_grads=True, perturb=True):
    d = synthetic.make_mlp_inputs(B, NH, NC, 16, F, FF, seed=seed, eta_mode=eta_mode)
    if perturb:
        d = synthetic.perturb_params(d, seed=seed + 7)
    d = {k: v.float() for k, v in d.items()}
    d64 = {k: v.double() for k, v in d.items()}

    def fn(XQ, XK, XV, eta, ln_w, ln_b, W1, b1, W2, b2):
        return ref_ops.ttt_mlp(XK, XQ, XV, eta, ln_w, ln_b, W1, b1, W2, b2, ckpt)

    leaves = {k: d64[k] for k in ("XQ", "XK", "XV", "eta", "ln_w", "ln_b", "W1", "b1", "W2", "b2")}
    res = {("in_" + k): _np(v) for k, v in d.items()}
    res["ckpt"] = np.array(ckpt)
    if with_grads:
        dO = synthetic.make_upstream((B, NC, 16, NH, F), seed=seed + 1).double()
        out, grads = _grads(fn, leaves, dO)
        res["dO"] = _np(dO)
        res.update({("grad_" + k): _np(v) for k, v in grads.items()})
    else:
        with torch.no_grad():
            out = fn(**leaves)
    res["out"] = _np(out)
    return res


def cached_readout_case(ref_root, NCs, F, FF, seed):
    sys.path.insert(0, ref_root)
    from kernels.mlp_cached_readout import mlp_cached_readout_kernel

    g = torch.Generator().manual_seed(seed)
    XQ = torch.randn(1, 1, NCs, 16, F, generator=g) / 8
    W1 = torch.randn(1, 1, F, FF, generator=g) * 0.05
    b1 = torch.randn(1, 1, 1, FF, generator=g) * 0.02
    W2 = torch.randn(1, 1, FF, F, generator=g) * 0.05
    b2 = torch.randn(1, 1, 1, F, generator=g) * 0.02
    ln_w = 1 + 0.1 * torch.randn(1, F, generator=g)
    ln_b = 0.1 * torch.randn(1, F, generator=g)
    out = torch.empty(1, 1, NCs, 16, F)
    # the wrapper asserts CUDA tensors (kernels/mlp_cached_readout.py:122); the kernel
    # itself runs under the interpreter, launched as the wrapper does (:128-141)
    mlp_cached_readout_kernel[(1, 1, NCs)](
        XQ, W1, b1, W2, b2, ln_w, ln_b, out,
        CS_F_stride=16 * F, F_FF_stride=F * FF, FF_F_stride=FF * F, F_stride=F, FF_stride=FF,
        NH=1, CS=16, F=F, FF=FF, num_warps=4,
    )
    res = {"in_XQ": XQ, "in_W1": W1, "in_b1": b1, "in_W2": W2, "in_b2": b2, "in_ln_w": ln_w, "in_ln_b": ln_b, "out": XQ + out}
    return {k: _np(v) for k, v in res.items()}


def memo_mix_case(ref_root, NC, F, FF, M, seed):
    """The reference's own memo-mixing loop (TTTMLP.ttt, ttt_layer.py:451-561) at B = NH = 1:
    TritonMLP.apply is stubbed to return the given scan output and memo states, and the
    cached read-outs run the reference's Triton kernel under the CPU interpreter (its CUDA
    wrapper is swapped for a launch of the same kernel). Gradients w.r.t. XQW, XU and XK
    come from autograd through the reference code."""
    import types

    sys.path.insert(0, ref_root)
    import ttt_layer
    from kernels.mlp_cached_readout import mlp_cached_readout_kernel

    NS = -(-NC // M)
    g = torch.Generator().manual_seed(seed)
    t = {
        "XQW": torch.randn(1, 1, NC, 16, F, generator=g) / 4,
        "XQ": torch.randn(1, 1, NC, 16, F, generator=g) / 8,
        "XK": torch.randn(1, 1, NC, 16, F, generator=g) / 8,
        "XU": torch.randn(1, 1, NC, 16, F, generator=g),
        "W1_memo": torch.randn(1, 1, NS, F, FF, generator=g) * 0.05,
        "b1_memo": torch.randn(1, 1, NS, 1, FF, generator=g) * 0.02,
        "W2_memo": torch.randn(1, 1, NS, FF, F, generator=g) * 0.05,
        "b2_memo": torch.randn(1, 1, NS, 1, F, generator=g) * 0.02,
        "ln_w": 1 + 0.1 * torch.randn(1, F, generator=g),
        "ln_b": 0.1 * torch.randn(1, F, generator=g),
    }
    dO = torch.randn(1, NC * 16, F, generator=g)
    leaves = {k: t[k].clone().requires_grad_(True) for k in ("XQW", "XU", "XK")}

    def readout(XQ_seg, W1, b1, W2, b2, ln_w, ln_b):
        XQ_seg, W1, b1, W2, b2 = (x.detach().contiguous() for x in (XQ_seg, W1, b1, W2, b2))
        out = torch.empty_like(XQ_seg)
        mlp_cached_readout_kernel[(1, 1, XQ_seg.shape[2])](
            XQ_seg, W1, b1, W2, b2, ln_w.detach(), ln_b.detach(), out,
            CS_F_stride=16 * F, F_FF_stride=F * FF, FF_F_stride=FF * F, F_stride=F, FF_stride=FF,
            NH=1, CS=16, F=F, FF=FF, num_warps=4,
        )
        return XQ_seg + out

    class StubMLP:
        # The scan output is handed over in a non-contiguous layout: with B = NH = 1 a
        # contiguous one would make the loop's `.contiguous()` segment copies (ttt_layer.py:516)
        # aliases of the tensor it then writes in place (:557), which autograd rejects; with
        # B * NH > 1, as in training, the slices are strided and copied anyway.
        @staticmethod
        def apply(*args):
            xqw = leaves["XQW"].transpose(-1, -2).contiguous().transpose(-1, -2)
            return (xqw, t["W1_memo"], t["b1_memo"], t["W2_memo"], t["b2_memo"])

    saved = ttt_layer.mlp_cached_readout_triton, ttt_layer.TritonMLP
    ttt_layer.mlp_cached_readout_triton, ttt_layer.TritonMLP = readout, StubMLP
    try:
        layer = types.SimpleNamespace(
            W1=torch.zeros(1, F, FF), b1=torch.zeros(1, 1, FF), W2=torch.zeros(1, FF, F), b2=torch.zeros(1, 1, F),
            ttt_norm_weight=t["ln_w"], ttt_norm_bias=t["ln_b"], use_kernel=True, width=F,
            config=types.SimpleNamespace(scan_checkpoint_group_size=1, mem_cache_segment_n_mini_batches=M))
        inputs = {"XQ": t["XQ"], "XK": leaves["XK"], "XV": t["XQ"], "XU": leaves["XU"],
                  "eta": torch.zeros(1, 1, NC, 16, 16)}
        out = ttt_layer.TTTMLP.ttt(layer, inputs)  # [B, L, NH * F]
        out.backward(dO)
    finally:
        ttt_layer.mlp_cached_readout_triton, ttt_layer.TritonMLP = saved
    res = {"in_" + k: v for k, v in t.items()}
    res.update({"M": torch.tensor(M), "dO": dO.reshape(1, NC, 16, 1, F).permute(0, 3, 1, 2, 4),
                "out": out.detach().reshape(1, NC, 16, 1, F).permute(0, 3, 1, 2, 4)})
    res.update({"grad_" + k: v.grad for k, v in leaves.items()})
    return {k: _np(v) for k, v in res.items()}


def prologue_case(ref_root, B, L, W, NH, CS, seed):
    """The reference layer's own input prologue: TTTMLP.process_input (ttt_layer.py:261-330)
    of a TTTWrapper built from a ModelConfig, eager (TorchDynamo disabled), float64, with
    autograd gradients of every input. freqs_cis is the wrapper's own buffer."""
    sys.path.insert(0, ref_root)
    import forecast
    import ttt_layer

    torch.manual_seed(seed)
    cfg = forecast.ModelConfig(seq_len=L, model_dim=W, num_heads=NH, mini_batch_size=CS, ssm_layer="ttt_mlp",
                               use_kernel=False, ttt_base_lr=0.1)
    wrapper = ttt_layer.TTTWrapper(cfg).double()
    layer = wrapper.ttt
    with torch.no_grad():  # non-trivial gate and LN parameters
        layer.learnable_ttt_lr_bias.normal_(0, 0.5)
        layer.ttt_norm_weight.add_(0.1 * torch.randn_like(layer.ttt_norm_weight))
        layer.ttt_norm_bias.add_(0.1 * torch.randn_like(layer.ttt_norm_bias))
    hidden = torch.randn(B, L, W, dtype=torch.float64, requires_grad=True)
    out = layer.process_input(hidden, wrapper.freqs_cis, forecast.SequenceMetadata())
    g = torch.Generator().manual_seed(seed + 1)
    douts = {k: torch.randn(out[k].shape, generator=g, dtype=torch.float64) for k in ("XQ", "XK", "XV", "XU", "eta")}
    loss = sum((out[k] * douts[k]).sum() for k in douts)
    loss.backward()
    fc = wrapper.freqs_cis[:L]
    res = {
        "in_hidden": hidden.detach(), "in_wq": layer.wq.weight, "in_bq": layer.wq.bias, "in_wk": layer.wk.weight,
        "in_bk": layer.wk.bias, "in_wv": layer.wv.weight, "in_bv": layer.wv.bias, "in_wu": layer.wu.weight,
        "in_bu": layer.wu.bias, "in_lr_w": layer.learnable_ttt_lr_weight, "in_lr_b": layer.learnable_ttt_lr_bias,
        "in_ln_w": layer.ttt_norm_weight, "in_ln_b": layer.ttt_norm_bias,
        "in_freqs_cos": fc.real, "in_freqs_sin": fc.imag, "CS": torch.tensor(CS), "base_lr": torch.tensor(0.1),
    }
    res.update({"out_" + k: v for k, v in out.items()})
    res.update({"d_" + k: v for k, v in douts.items()})
    grads = {"hidden": hidden.grad, "wq": layer.wq.weight.grad, "bq": layer.wq.bias.grad,
             "wk": layer.wk.weight.grad, "bk": layer.wk.bias.grad, "wv": layer.wv.weight.grad,
             "bv": layer.wv.bias.grad, "wu": layer.wu.weight.grad, "bu": layer.wu.bias.grad,
             "lr_w": layer.learnable_ttt_lr_weight.grad, "lr_b": layer.learnable_ttt_lr_bias.grad,
             "ln_w": layer.ttt_norm_weight.grad, "ln_b": layer.ttt_norm_bias.grad}
    res.update({"grad_" + k: v for k, v in grads.items()})
    return {k: _np(v) for k, v in res.items()}


def epilogue_case(ref_root, B, L, W, NH, CS, seed):
    """The reference layer's own output epilogue: TTTBase.forward (ttt_layer.py:337-357) of a
    TTTWrapper built from a ModelConfig, float64, with its ttt() replaced by a stub that
    returns a given scan output XQW [B, NH, NC, CS, F] through TTTMLP.ttt's own tail
    (permute(0, 2, 3, 1, 4) + reshape, :563-564); post_norm and wo are the layer's modules."""
    sys.path.insert(0, ref_root)
    import forecast
    import ttt_layer

    torch.manual_seed(seed)
    cfg = forecast.ModelConfig(seq_len=L, model_dim=W, num_heads=NH, mini_batch_size=CS, ssm_layer="ttt_mlp",
                               use_kernel=False)
    wrapper = ttt_layer.TTTWrapper(cfg).double()
    layer = wrapper.ttt
    with torch.no_grad():
        layer.post_norm.weight.add_(0.1 * torch.randn_like(layer.post_norm.weight))
        layer.post_norm.bias.add_(0.1 * torch.randn_like(layer.post_norm.bias))
    F, NC = W // NH, L // CS
    XQW = torch.randn(B, NH, NC, CS, F, dtype=torch.float64, requires_grad=True)
    layer.ttt = lambda inputs: XQW.permute(0, 2, 3, 1, 4).reshape(B, L, W)
    hidden = torch.randn(B, L, W, dtype=torch.float64)
    out = layer(hidden, wrapper.freqs_cis, forecast.SequenceMetadata())
    dout = torch.randn(out.shape, generator=torch.Generator().manual_seed(seed + 1), dtype=torch.float64)
    (out * dout).sum().backward()
    res = {"in_XQW": XQW.detach(), "in_pn_w": layer.post_norm.weight, "in_pn_b": layer.post_norm.bias,
           "in_wo_w": layer.wo.weight, "in_wo_b": layer.wo.bias, "out": out.detach(), "dout": dout,
           "eps": torch.tensor(layer.post_norm.eps), "grad_XQW": XQW.grad, "grad_pn_w": layer.post_norm.weight.grad,
           "grad_pn_b": layer.post_norm.bias.grad, "grad_wo_w": layer.wo.weight.grad, "grad_wo_b": layer.wo.bias.grad}
    return {k: _np(v) for k, v in res.items()}


def forecaster_case(ref_root, B, L, W, NH, CS, pred_len, d_in, seed):
    """The reference's own TTTForecaster (forecast.py:79-99, one TTT-MLP layer, use_kernel
    path) in float64 with MSE loss, gradients of every parameter. Its TritonMLP launch is
    replaced by the reference's ops.ttt_mlp, returned in the kernel layout [B, NH, NC, CS, F]
    the Triton kernel writes (ops returns [B, NC, CS, NH, F]); one memo segment covers the
    sequence, so the mixing loop passes the scan output through (no cached read-outs)."""
    sys.path.insert(0, ref_root)
    import forecast
    import ops as ref_ops
    import ttt_layer

    class ScanStub:
        @staticmethod
        def apply(ln_w, ln_b, W1, b1, W2, b2, XQ, XV, XK, eta, ckpt, memo):
            out = ref_ops.ttt_mlp(XK, XQ, XV, eta, ln_w, ln_b, W1, b1, W2, b2, ckpt)
            return out.permute(0, 3, 1, 2, 4), None, None, None, None

    torch.manual_seed(seed)
    NC = L // CS
    cfg = forecast.ModelConfig(seq_len=L, model_dim=W, num_heads=NH, mini_batch_size=CS, ssm_layer="ttt_mlp",
                               use_kernel=True, ttt_base_lr=0.1, scan_checkpoint_group_size=2,
                               mem_cache_segment_n_mini_batches=NC)
    saved = ttt_layer.TritonMLP
    ttt_layer.TritonMLP = ScanStub
    try:
        model = forecast.TTTForecaster(cfg, d_in=d_in, d_out=d_in, pred_len=pred_len).double()
        with torch.no_grad():  # non-trivial gate, LayerNorm and inner-bias parameters
            layer = model.ttt.ttt
            layer.learnable_ttt_lr_bias.normal_(0, 0.5)
            for t in (layer.ttt_norm_weight, layer.post_norm.weight):
                t.add_(0.1 * torch.randn_like(t))
            for t in (layer.ttt_norm_bias, layer.post_norm.bias, layer.b1, layer.b2):
                t.normal_(0, 0.05)
        x = torch.randn(B, L, d_in, dtype=torch.float64)
        y = torch.randn(B, pred_len, d_in, dtype=torch.float64)
        out = model(x)
        loss = torch.nn.functional.mse_loss(out, y)
        loss.backward()
    finally:
        ttt_layer.TritonMLP = saved
    res = {"in_x": x, "in_y": y, "out": out.detach(), "loss": loss.detach(), "CS": torch.tensor(CS),
           "pred_len": torch.tensor(pred_len), "NH": torch.tensor(NH), "ckpt": torch.tensor(2),
           "memo": torch.tensor(NC), "base_lr": torch.tensor(0.1)}
    for k, v in model.state_dict().items():
        res["p_" + k] = v
    for k, v in model.named_parameters():  # wu gets no gradient with one memo segment: zeros
        res["g_" + k] = v.grad if v.grad is not None else torch.zeros_like(v)
    return {k: _np(v) for k, v in res.items()}


def forecaster_main_case(ref_root, B, W, NH, memo, seed):
    """The reference's TTTForecaster built from main.py's own ModelConfig (main.py:54-65: seq_len
    384, mini_batch_size 64, ttt_base_lr 0.05, checkpoint group 16, ttt_mlp with its F x F
    inner MLP, d_in = d_out = 1 for the univariate "S" features, pred_len 96) in float64 with
    MSE loss and the gradient of every parameter.

    The layer's TritonMLP launch runs the reference's own dual-form step
    (ops/ttt_mlp.py:compute_mini_batch) mini-batch by mini-batch, and its memo states are the
    states after mini-batch i for i % memo == 0 (the definition of kernels/mlp_forward.py:
    193-226), non-differentiable as mlp_triton.py:196 marks them. With memo < NC the layer's
    mixing loop runs the reference's cached read-out kernel under the CPU interpreter, which
    addresses only (b, h) = (0, 0) correctly (kernels/mlp_cached_readout.py:66-70), so that case
    uses B = NH = 1 (model_dim 32 keeps main.py's head_dim 32)."""
    sys.path.insert(0, ref_root)
    import forecast
    import ttt_layer
    from kernels.mlp_cached_readout import mlp_cached_readout_kernel
    from ops.ttt_mlp import compute_mini_batch

    L, CS, pred_len, d_in = 384, 64, 96, 1
    NC = L // CS
    memo = NC if memo is None else memo
    if memo < NC and B * NH != 1:
        raise ValueError("the reference's cached read-out kernel is correct only for B = NH = 1")

    class ScanStep:
        @staticmethod
        def apply(ln_w, ln_b, W1, b1, W2, b2, XQ, XV, XK, eta, ckpt, memo_seg):
            params = {"W1_states": W1, "b1_states": b1, "W2_states": W2, "b2_states": b2,
                      "ttt_norm_weight": ln_w, "ttt_norm_bias": ln_b}
            outs, mem = [], {k: [] for k in ("W1_states", "b1_states", "W2_states", "b2_states")}
            for n in range(XQ.shape[2]):
                x = {"XQ": XQ[:, :, n], "XV": XV[:, :, n], "XK": XK[:, :, n], "eta": eta[:, :, n]}
                params, o = compute_mini_batch(params, x)
                outs.append(o)
                if n % memo_seg == 0:
                    for k in mem:
                        mem[k].append(params[k].detach())
            memo_t = [torch.stack(mem[k], dim=2) for k in ("W1_states", "b1_states", "W2_states", "b2_states")]
            # handed over non-contiguous, as in memo_mix_case: with B = NH = 1 a contiguous
            # output makes the mixing loop's segment copies aliases it writes in place
            xqw = torch.stack(outs, dim=2).transpose(-1, -2).contiguous().transpose(-1, -2)
            return (xqw, *memo_t)

    def readout(XQ_seg, W1, b1, W2, b2, ln_w, ln_b):
        Bq, NHq, NCs, CSq, F = XQ_seg.shape
        FF = W1.shape[-1]
        XQ_seg, W1, b1, W2, b2 = (x.detach().contiguous() for x in (XQ_seg, W1, b1, W2, b2))
        out = torch.empty_like(XQ_seg)
        mlp_cached_readout_kernel[(1, 1, NCs)](
            XQ_seg, W1, b1, W2, b2, ln_w.detach(), ln_b.detach(), out,
            CS_F_stride=CSq * F, F_FF_stride=F * FF, FF_F_stride=FF * F, F_stride=F, FF_stride=FF,
            NH=1, CS=CSq, F=F, FF=FF, num_warps=4,
        )
        return XQ_seg + out

    torch.manual_seed(seed)
    cfg = forecast.ModelConfig(seq_len=L, model_dim=W, num_heads=NH, num_layers=1, ssm_layer="ttt_mlp",
                               mini_batch_size=CS, ttt_base_lr=0.05, scan_checkpoint_group_size=16,
                               latent_height=1, latent_width=1, compressed_num_frames=None,
                               mem_cache_segment_n_mini_batches=memo)
    saved = ttt_layer.TritonMLP, ttt_layer.mlp_cached_readout_triton
    ttt_layer.TritonMLP, ttt_layer.mlp_cached_readout_triton = ScanStep, readout
    try:
        model = forecast.TTTForecaster(cfg, d_in=d_in, d_out=d_in, pred_len=pred_len).double()
        with torch.no_grad():  # non-trivial gate, LayerNorm and inner-bias parameters
            layer = model.ttt.ttt
            layer.learnable_ttt_lr_bias.normal_(0, 0.5)
            for t in (layer.ttt_norm_weight, layer.post_norm.weight):
                t.add_(0.1 * torch.randn_like(t))
            for t in (layer.ttt_norm_bias, layer.post_norm.bias, layer.b1, layer.b2):
                t.normal_(0, 0.05)
        x = torch.randn(B, L, d_in, dtype=torch.float64)
        y = torch.randn(B, pred_len, d_in, dtype=torch.float64)
        out = model(x)
        loss = torch.nn.functional.mse_loss(out, y)
        loss.backward()
    finally:
        ttt_layer.TritonMLP, ttt_layer.mlp_cached_readout_triton = saved
    res = {"in_x": x, "in_y": y, "out": out.detach(), "loss": loss.detach(), "CS": torch.tensor(CS),
           "pred_len": torch.tensor(pred_len), "NH": torch.tensor(NH), "ckpt": torch.tensor(16),
           "memo": torch.tensor(memo), "base_lr": torch.tensor(0.05)}
    for k, v in model.state_dict().items():
        res["p_" + k] = v
    for k, v in model.named_parameters():  # wu gets no gradient with one memo segment: zeros
        res["g_" + k] = v.grad if v.grad is not None else torch.zeros_like(v)
    return {k: _np(v) for k, v in res.items()}


def main():
    if len(sys.argv) < 2:
        raise SystemExit("usage: python tests/golden/make_golden.py /path/to/ttt-triton")
    ref_root = sys.argv[1]
    sys.path.insert(0, ref_root)
    import forecast  # noqa: F401  (must precede ttt_layer / ops imports in the reference)
    import ops as ref_ops

    cases = {
        "linear_small": lambda: linear_case(ref_ops, B=2, NH=2, NC=4, F=32, ckpt=2, eta_mode="causal", seed=10),
        "linear_equal_eta": lambda: linear_case(ref_ops, B=1, NH=2, NC=3, F=64, ckpt=16, eta_mode="equal", seed=11),
        "linear_config0_fwd": lambda: linear_case(ref_ops, B=2, NH=4, NC=16, F=64, ckpt=16, eta_mode="causal", seed=0, with_grads=False, perturb=False),
        "mlp_small": lambda: mlp_case(ref_ops, B=2, NH=2, NC=3, F=16, FF=64, ckpt=2, eta_mode="causal", seed=20),
        "mlp_fxf_equal_eta": lambda: mlp_case(ref_ops, B=1, NH=2, NC=3, F=32, FF=32, ckpt=16, eta_mode="equal", seed=21),
        "cached_readout": lambda: cached_readout_case(ref_root, NCs=3, F=32, FF=128, seed=30),
        "memo_mix": lambda: memo_mix_case(ref_root, NC=7, F=32, FF=128, M=2, seed=40),
        "prologue": lambda: prologue_case(ref_root, B=2, L=64, W=128, NH=2, CS=16, seed=50),
        "epilogue": lambda: epilogue_case(ref_root, B=2, L=32, W=128, NH=4, CS=16, seed=60),
        "forecaster": lambda: forecaster_case(ref_root, B=2, L=64, W=128, NH=2, CS=16, pred_len=8, d_in=7, seed=70),
        # main.py's own model configuration (CS 64, head_dim 32, F x F inner MLP)
        "forecaster_main": lambda: forecaster_main_case(ref_root, B=2, W=128, NH=4, memo=None, seed=80),
        "forecaster_main_memo": lambda: forecaster_main_case(ref_root, B=1, W=32, NH=1, memo=2, seed=81),
    }
    only = sys.argv[2:]  # optional case names: regenerate just those
    if only:
        cases = {k: v for k, v in cases.items() if k in only}
    for name, make in cases.items():
        res = make()
        path = os.path.join(HERE, name + ".npz")
        np.savez_compressed(path, **res)
        print(f"wrote {path} ({os.path.getsize(path) / 1024:.0f} KiB)")


if __name__ == "__main__":
    main()
