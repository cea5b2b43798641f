"""Benchmark of the B200 TTT dual-form scan (one JSON line from rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]
    torchrun --nproc-per-node N bench.py --gpus N ...        (N > 1)

Workloads (synthetic seeded data of those shapes, see
ttt-triton_b200/synthetic.py):

* ``mlp_fwd_c1`` (default, the headline): TTT-MLP forward, B16 NH12 L2048 F64 FF256,
  bf16 activations / fp32 state, checkpoint group 16 (config 1).
* ``linear_fwd_c0``: TTT-Linear forward, fp32, B2 NH4 L256 F64 (config 0).
* ``linear_fwd_c2``: TTT-Linear forward only at the config-2 shape (diagnostic).
* ``linear_fwdbwd_c2``: TTT-Linear forward+backward, bf16, B32 NH8 L4096 F64 (config 2).
* ``mlp_fwdbwd_c3``: TTT-MLP forward+backward, bf16, B64 NH16 L8192 F64 FF256, memo 16 (config 3).
* ``memo_mix_c3``: the layer's memo-state mixing (cached read-outs of every earlier memo
  state, ttt_layer.py:503-559), forward+backward, at the config-3 shape (32 memo segments).
* ``prologue_c4``: one TTT layer's input prologue (process_input, ttt_layer.py:261-330:
  projections, L2 norm, rotary embedding, LN target, eta), forward+backward, bf16, at the
  config-4 forecaster shape (global batch 256, lookback 336, d_model 256, 4 heads).
* ``epilogue_c4``: the layer's output epilogue (scan output -> post_norm -> wo,
  ttt_layer.py:349-350, 563-564), forward+backward, bf16, at the same shape.
* ``forecaster_c4``: one training step of the config-4 forecaster (4 TTT-MLP layers,
  d_model 256, 4 heads, mini-batch 16, F x F inner MLP, memo segments of 2 mini-batches;
  lookback 336, horizon 96, 7 channels, global batch 256, MSE, AdamW, clipping), every TTT
  stage on this library, bf16 activations. Strong scaling: the global batch is split over
  the ranks and DistributedDataParallel averages the gradients with NCCL.
* ``forecaster_main``: one training step of the reference's own main.py model (one TTT-MLP
  layer, d_model 128, 4 heads of 32, mini-batch 64, base learning rate 0.05, lookback 384,
  horizon 96, one channel, batch 32, fp16 activations), on the general kernels.

A step is one pass of the hot path over one batch. Multi-GPU runs of a workload are weak
scaling: every rank processes its own full batch (the (b, h) streams are independent, so
there is no data-path collective); timing is the max over ranks of the device-timed region.

The default line (``mlp_fwd_c1``) also carries two training records, ``fwdbwd`` (config 3:
TTT-MLP forward+backward, B64 NH16 L8192) and ``fwdbwd_linear`` (config 2: TTT-Linear
forward+backward, B32 NH8 L4096), each as ONE global batch whose (batch, head) streams are
split over the ranks by batch (sharding.py), strong scaling: at N GPUs each rank runs B/N
batches, the step time is the max over ranks and the value is the global tokens over it.
Each has its own roofline (the backward kernel), end-to-end leg and CPU baseline.

The reference arm (``--impl reference``) times the CPU port of the reference's ops/ path
(oracle/ttt_oracle.py) on the host cores at the workload's full shape (chunked over
streams); the training workloads and the forecaster run a bounded batch slice there.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "ttt-triton_b200"))

import torch  # noqa: E402

WORKLOADS = {
    "linear_fwd_c0": dict(kind="linear", B=2, NH=4, L=256, F=64, FF=None, dtype="f32", bwd=False, ckpt=16, memo=None),
    "mlp_fwd_c1": dict(kind="mlp", B=16, NH=12, L=2048, F=64, FF=256, dtype="bf16", bwd=False, ckpt=16, memo=None),
    "linear_fwd_c2": dict(kind="linear", B=32, NH=8, L=4096, F=64, FF=None, dtype="bf16", bwd=False, ckpt=16, memo=None),
    "linear_fwdbwd_c2": dict(kind="linear", B=32, NH=8, L=4096, F=64, FF=None, dtype="bf16", bwd=True, ckpt=16, memo=None),
    "mlp_fwdbwd_c3": dict(kind="mlp", B=64, NH=16, L=8192, F=64, FF=256, dtype="bf16", bwd=True, ckpt=16, memo=16),
    "memo_mix_c3": dict(kind="memo", B=64, NH=16, L=8192, F=64, FF=256, dtype="bf16", bwd=True, ckpt=16, memo=16),
    "prologue_c4": dict(kind="prologue", B=256, NH=4, L=336, F=64, FF=None, dtype="bf16", bwd=True, ckpt=None,
                        memo=None),
    "epilogue_c4": dict(kind="epilogue", B=256, NH=4, L=336, F=64, FF=None, dtype="bf16", bwd=True, ckpt=None,
                        memo=None),
    "forecaster_c4": dict(kind="forecaster", B=256, NH=4, L=336, F=64, FF=64, dtype="bf16", bwd=True, ckpt=16,
                          memo=2, layers=4, horizon=96, channels=7),
    # the reference's own main.py model: ModelConfig(seq_len=384, model_dim=128, num_heads=4,
    # mini_batch_size=64, ttt_base_lr=0.05, ...), batch 32, univariate series, fp16 autocast
    "forecaster_main": dict(kind="forecaster", B=32, NH=4, L=384, F=32, FF=32, dtype="f16", bwd=True, ckpt=16,
                            memo=2, layers=1, horizon=96, channels=1, cs=64, base_lr=0.05),
}
MEMO = ("XQW", "XQ", "XK", "XU", "W1_memo", "b1_memo", "W2_memo", "b2_memo", "ln_w", "ln_b")
PRO = ("hidden", "wq", "bq", "wk", "bk", "wv", "bv", "wu", "bu", "lr_w", "lr_b", "ln_w", "ln_b")
PRO_OUTS = ("XQ", "XK", "XV", "XU", "eta")
BASE_LR = 0.1  # forecast.ModelConfig.ttt_base_lr
EPI = ("XQW", "pn_w", "pn_b", "wo_w", "wo_b")
POST_NORM_EPS = 1e-6  # ttt_layer.py:77
RESULT_KEY = {"prologue": "hidden", "epilogue": "XQW"}  # the input whose gradient e2e reads back
CS = 16
DT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}
# DRAM bytes (read + write) of one call of the dominant kernel's entry point from an ncu
# capture of the same workload: (bytes, tokens in that call, summary file). Scaled to the
# call measured here by tokens processed. The config-1 forward is two launches (the
# balanced schedule); its bytes are their sum.
NCU_TRAFFIC = {
    ("mlp_fwd_c1", "mlp_fwd"): (270.5e6, 16 * 12 * 2048, "profiles/mlp_fwd_tc_config1.md"),
    ("linear_fwd_c2", "linear_fwd"): (557.3e6, 32 * 8 * 4096, "profiles/linear_fwd_tc_config2.md"),
    ("linear_fwdbwd_c2", "linear_bwd"): (1252.9e6, 32 * 8 * 4096, "profiles/linear_bwd_tc_config2.md"),
    # captured at batch 4 (64 streams); traffic per stream is size-independent, scaled by tokens
    ("mlp_fwdbwd_c3", "mlp_bwd"): (1851.7e6, 4 * 16 * 8192, "profiles/mlp_bwd_tc_config3.md"),
}
METRIC = "TTT tokens/s (B*H*L) fwd & fwd+bwd at 1/2/4/8 B200; % of HBM roofline"


def peaks():
    path = os.path.join(HERE, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, 1400.0, "fallback"


def algorithmic(w):
    """Compulsory bytes and useful FLOPs per token (one (b, h, t)) for each pass.

    Bytes: the forward reads XQ, XK, XV and one eta row and writes XQW; the backward
    re-reads those inputs, reads dXQW and writes dXQ, dXK, dXV and one eta row of d_eta.
    Inner state, checkpoints, memo states and the stored pre-activations are excluded.
    FLOPs: 2 * (multiply-adds) of the dual-form products of ops/ttt_linear.py:8-54 /
    ops/ttt_mlp.py:9-67 and of their hand-derived backward (reverse walk over stored Z).
    """
    F, FF = w["F"], w["FF"]
    eb = 4 if w["dtype"] == "f32" else 2
    if w["kind"] == "prologue":
        # Per (token, head): the element-wise forward reads the head's projection segment
        # (q, k, v, u and the gate: 4F + 1) and writes XQ, XK, XV, XU and its eta column (CS
        # rows); the backward reads that segment, dXQ, dXK, dXV, dXU and the d_eta column and
        # writes d proj. FLOPs are the projection GEMMs: 2 * W * (4F + 1) forward, twice that
        # backward (d hidden and d weights), W = NH * F.
        Wd = w["NH"] * F
        return {"fwd": (eb * (8 * F + 1 + CS), 2 * Wd * (4 * F + 1)),
                "bwd": (eb * (12 * F + 2 + CS), 4 * Wd * (4 * F + 1))}
    if w["kind"] == "epilogue":
        # Per (token, head): the forward kernel reads the head's F scan outputs and writes F
        # normalised values; the backward reads them again with F of d(normalised) and F of
        # d out (for the wo bias gradient) and writes F of d XQW. FLOPs are the wo GEMMs:
        # 2 * W * F forward, twice that backward.
        Wd = w["NH"] * F
        return {"fwd": (eb * 2 * F, 2 * Wd * F), "bwd": (eb * 4 * F, 4 * Wd * F)}
    if w["kind"] == "memo":
        # forward reads XQW, XQ, XK, XU and writes the output; backward re-reads XQW, XQ, XK,
        # XU, reads dOut and writes dXQW, dXU, dXK. Each token of segment i reads out the i
        # earlier memo states (2 * 2 * F * FF FLOPs each) in both passes.
        NC, M = w["L"] // CS, w["memo"]
        NS = -(-NC // M)
        mean_i = sum(i * (min((i + 1) * M, NC) - i * M) for i in range(NS)) / NC
        flops = mean_i * 4 * F * FF
        return {"fwd": (eb * 5 * F, flops), "bwd": (eb * 8 * F, flops)}
    fwd_bytes = eb * (3 * F + CS + F)
    bwd_bytes = eb * ((3 * F + CS) + F + (3 * F + CS))
    if w["kind"] == "linear":
        fwd_flops = 6 * F * F + 4 * CS * F
        bwd_flops = 16 * F * F + 12 * CS * F
    else:
        fwd_flops = 14 * F * FF + 4 * CS * F + 4 * CS * FF
        bwd_flops = 38 * F * FF + 12 * CS * FF + 12 * CS * F
    return {"fwd": (fwd_bytes, fwd_flops), "bwd": (bwd_bytes, bwd_flops)}


# --------------------------------------------------------------------------- inputs / steps
def make_inputs(w, device, seed):
    import synthetic as S

    NC = w["L"] // CS
    dt = DT[w["dtype"]]
    if w["kind"] == "prologue":
        d = S.make_prologue_inputs(w["B"], w["L"], w["NH"] * w["F"], w["NH"], device=device, seed=seed)
        d = {k: (v if k in ("ln_w", "ln_b", "freqs_cos", "freqs_sin") else v.to(dt)) for k, v in d.items()}
        shp = (w["B"], w["NH"], NC, CS, w["F"])
        dO = {k: S.make_upstream(shp if k != "eta" else shp[:-1] + (CS,), device=device, seed=seed + 1 + i, dtype=dt)
              for i, k in enumerate(PRO_OUTS)}
        return d, dO
    if w["kind"] == "epilogue":
        g = torch.Generator(device=device).manual_seed(seed)
        W = w["NH"] * w["F"]
        d = {"XQW": (torch.randn(w["B"], w["NH"], NC, CS, w["F"], generator=g, device=device) * 0.5).to(dt),
             "pn_w": 1 + 0.1 * torch.randn(W, generator=g, device=device),
             "pn_b": 0.1 * torch.randn(W, generator=g, device=device),
             "wo_w": (0.02 * torch.randn(W, W, generator=g, device=device)).to(dt),
             "wo_b": (0.02 * torch.randn(W, generator=g, device=device)).to(dt)}
        return d, S.make_upstream((w["B"], w["L"], W), device=device, seed=seed + 1, dtype=dt)
    if w["kind"] == "memo":
        return S.make_memo_inputs(w["B"], w["NH"], NC, CS, w["F"], w["FF"], w["memo"], dtype=dt, device=device,
                                  seed=seed), S.make_upstream((w["B"], w["NH"], NC, CS, w["F"]), device=device,
                                                              seed=seed + 1, dtype=dt)
    if w["kind"] == "linear":
        d = S.make_linear_inputs(w["B"], w["NH"], NC, CS, w["F"], dtype=dt, device=device, seed=seed)
    else:
        d = S.make_mlp_inputs(w["B"], w["NH"], NC, CS, w["F"], w["FF"], dtype=dt, device=device, seed=seed)
    dO = S.make_upstream((w["B"], w["NH"], NC, CS, w["F"]), device=device, seed=seed + 1, dtype=dt) if w["bwd"] else None
    return d, dO


LIN = ("ln_w", "ln_b", "W1", "b1", "XQ", "XV", "XK", "eta")
MLP = ("ln_w", "ln_b", "W1", "b1", "W2", "b2", "XQ", "XV", "XK", "eta")


def kernel_step(w, d, dO):
    """One pass of the hot path through the functional core (inputs resident in HBM).
    Returns the number of the library's kernels it launched (its own launch counter)."""
    import _core
    import _lib

    n0 = _lib.launch_count()
    if w["kind"] == "prologue":
        prologue_step(w, d, dO)
    elif w["kind"] == "epilogue":
        epilogue_step(w, d, dO)
    elif w["kind"] == "memo":
        _core.memo_mix_forward(*(d[k] for k in MEMO), w["memo"])
        if w["bwd"]:
            _core.memo_mix_backward(*(d[k] for k in MEMO), w["memo"], dO)
    elif w["kind"] == "linear":
        XQW, Wl, bl, Wc, bc, Z = _core.linear_forward(*(d[k] for k in LIN), w["ckpt"], for_backward=w["bwd"])
        if w["bwd"]:
            _core.linear_backward(d["ln_w"], d["ln_b"], Wc, bc, d["XQ"], d["XV"], d["XK"], d["eta"], dO, w["ckpt"],
                                  Z=Z, W_last=Wl, b_last=bl)
    else:
        XQW, last, ck, _, zs = _core.mlp_forward(*(d[k] for k in MLP), w["ckpt"], memo_of(w), for_backward=w["bwd"])
        if w["bwd"]:
            _core.mlp_backward(d["ln_w"], d["ln_b"], ck, d["XQ"], d["XV"], d["XK"], d["eta"], dO, w["ckpt"],
                               saved=zs, W1_last=last[0], W2_last=last[2])
    return _lib.launch_count() - n0


def memo_of(w):
    """Memo-segment size of an MLP workload. TritonMLP.apply always writes memo states
    (mlp_triton.py:15-62), so the device-timed and the end-to-end legs both ask for them: at
    the workload's memo size, or, for a workload that names none (config 1), one segment
    covering the sequence, the API's minimum (one memo state per stream)."""
    return w["memo"] or w["L"] // CS


def prologue_step(w, d, dO):
    """Forward and backward of the prologue through the functional core: the projection GEMM
    (library), the element-wise forward kernel, the element-wise backward kernel and the two
    projection-gradient GEMMs (library)."""
    import _core
    from prologue import concat_projections

    B, L, NH, F = w["B"], w["L"], w["NH"], w["F"]
    Wcat, bcat, _, _ = concat_projections(*(d[k] for k in PRO[1:11]))
    h2 = d["hidden"].reshape(B * L, -1)
    P = torch.addmm(bcat, h2, Wcat.t())
    scale = BASE_LR / (F * CS)
    _core.prologue_forward(P, B, L, NH, F, CS, d["ln_w"], d["ln_b"], d["freqs_cos"], d["freqs_sin"], scale)
    dP, _, _, _ = _core.prologue_backward(P, B, L, NH, F, CS, d["ln_w"], d["ln_b"], d["freqs_cos"],
                                          d["freqs_sin"], scale, *(dO[k] for k in PRO_OUTS))
    torch.mm(dP, Wcat)
    torch.mm(dP.t(), h2)


def epilogue_step(w, d, dO):
    """Forward and backward of the output epilogue through the functional core: post_norm
    kernel, wo GEMM (library), the two wo-gradient GEMMs and bias sum (library) and the
    post_norm backward kernel."""
    import _core

    Y = _core.post_norm_forward(d["XQW"], d["pn_w"], d["pn_b"], POST_NORM_EPS)
    torch.addmm(d["wo_b"], Y, d["wo_w"].t())
    d2 = dO.reshape(Y.shape)
    dY = torch.mm(d2, d["wo_w"])
    torch.mm(d2.t(), Y)
    _core.post_norm_backward(d["XQW"], d["pn_w"], d["pn_b"], POST_NORM_EPS, dY, d2)


def api_compute(w, d):
    """One step through the public API on device buffers d (the reference-facing call:
    TritonLinear / TritonMLP .apply, mlp_memo_mix, ttt_prologue or post_norm_wo, plus the
    backward for training workloads). Returns the device tensor the step reads back: the
    output, or the gradient of RESULT_KEY / XQ for training workloads."""
    from linear_triton import TritonLinear
    from mlp_triton import TritonMLP

    def grad_of(leaves, key):
        res = d[key].grad
        for t in leaves:
            t.grad = None
            t.requires_grad_(False)
        return res

    if w["kind"] == "prologue":
        from prologue import ttt_prologue

        leaves = [d[k].requires_grad_(True) for k in PRO]
        out = ttt_prologue(*leaves, (d["freqs_cos"], d["freqs_sin"]), CS, BASE_LR)
        torch.autograd.backward([out[k] for k in PRO_OUTS], [d["d_" + k] for k in PRO_OUTS])
        return grad_of(leaves, "hidden")
    if w["kind"] == "epilogue":
        from epilogue import post_norm_wo

        leaves = [d[k].requires_grad_(True) for k in EPI]
        post_norm_wo(*leaves, POST_NORM_EPS).backward(d["dO"])
        return grad_of(leaves, "XQW")
    if w["kind"] == "memo":
        from kernels.mlp_memo_mix import mlp_memo_mix

        leaves = [d[k].requires_grad_(k in ("XQW", "XU", "XK")) for k in MEMO]
        mlp_memo_mix(*leaves, w["memo"]).backward(d["dO"])
        return grad_of(leaves, "XU")
    if w["kind"] == "linear":
        leaves = [d[k].requires_grad_(w["bwd"]) for k in LIN]
        out = TritonLinear.apply(*leaves, w["ckpt"])
    else:
        leaves = [d[k].requires_grad_(w["bwd"]) for k in MLP]
        out = TritonMLP.apply(*leaves, w["ckpt"], memo_of(w))[0]
    if w["bwd"]:
        out.backward(d["dO"])
        return grad_of(leaves, "XQ")
    return out.detach()


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.file = None

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.file, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.2)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        with open(self.file.name) as f:
            rows = [r.split(",") for r in f.read().strip().splitlines() if r.strip()]
        os.unlink(self.file.name)
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            r = [x.strip() for x in r]
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                mx = max(mx, float(r[2]))
            except ValueError:
                continue
            for n, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def smi_index(dev):
    """nvidia-smi's index of a torch CUDA device (CUDA_VISIBLE_DEVICES renumbers devices)."""
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [x.strip() for x in vis.split(",") if x.strip()]
        if dev.index < len(ids) and ids[dev.index].isdigit():
            return int(ids[dev.index])
    return dev.index


# --------------------------------------------------------------------------- arms
def cpu_reference(w, budget_s=12.0):
    """The reference's ops/ path restated on the host cores (oracle/ttt_oracle.py), fp32,
    on a bounded sample of the workload: the full sequence for a batch slice."""
    sys.path.insert(0, os.path.join(HERE, "oracle"))
    import synthetic as S
    import ttt_oracle as O

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    NC = w["L"] // CS
    B, NH = 1, min(w["NH"], 4)
    if w["kind"] == "prologue":
        B = 32
        d = S.make_prologue_inputs(B, w["L"], w["NH"] * w["F"], w["NH"], seed=0)
        shp = (B, w["NH"], NC, CS, w["F"])
        dO = {k: S.make_upstream(shp if k != "eta" else shp[:-1] + (CS,), seed=1 + i) for i, k in enumerate(PRO_OUTS)}
        best, reps = None, 0
        t_end = time.perf_counter() + budget_s
        while reps < 1 or (time.perf_counter() < t_end and reps < 20):
            t0 = time.perf_counter()
            O.process_input_grads(d, dO, CS, BASE_LR)
            dt = time.perf_counter() - t0
            best = dt if best is None else min(best, dt)
            reps += 1
        sample = f"B={B} L={w['L']} W={w['NH'] * w['F']} NH={w['NH']} (batch slice), fp32, fwd+bwd, best of {reps}"
        return B * w["NH"] * w["L"] / best, threads, sample
    if w["kind"] == "epilogue":
        B = 32
        g = torch.Generator().manual_seed(0)
        W = w["NH"] * w["F"]
        d = {"XQW": torch.randn(B, w["NH"], NC, CS, w["F"], generator=g) * 0.5, "pn_w": torch.ones(W),
             "pn_b": torch.zeros(W), "wo_w": 0.02 * torch.randn(W, W, generator=g), "wo_b": torch.zeros(W)}
        dout = torch.randn(B, w["L"], W, generator=g)
        best, reps = None, 0
        t_end = time.perf_counter() + budget_s
        while reps < 1 or (time.perf_counter() < t_end and reps < 20):
            t0 = time.perf_counter()
            O.post_norm_wo_grads(d, dout)
            dt = time.perf_counter() - t0
            best = dt if best is None else min(best, dt)
            reps += 1
        sample = f"B={B} L={w['L']} W={W} NH={w['NH']} (batch slice), fp32, fwd+bwd, best of {reps}"
        return B * w["NH"] * w["L"] / best, threads, sample
    if w["kind"] == "memo":
        B, NH = 1, 1
        d = S.make_memo_inputs(B, NH, NC, CS, w["F"], w["FF"], w["memo"], seed=0)
        dO = S.make_upstream((B, NH, NC, CS, w["F"]), seed=1)
        tokens = B * NH * NC * CS
        t0 = time.perf_counter()
        O.memo_mix_grads(d, dO, w["memo"])
        dt = time.perf_counter() - t0
        return tokens / dt, threads, f"B=1 NH=1 L={w['L']} (full sequence, one stream), fp32, forward+backward, 1 run"
    if w["kind"] == "linear":
        d = S.make_linear_inputs(B, NH, NC, CS, w["F"], seed=0)
    else:
        d = S.make_mlp_inputs(B, NH, NC, CS, w["F"], w["FF"], seed=0)
    dO = S.make_upstream((B, NH, NC, CS, w["F"]), seed=1)
    tokens = B * NH * NC * CS
    best = None
    t_end = time.perf_counter() + budget_s
    reps = 0
    while reps < 1 or (time.perf_counter() < t_end and reps < 20):
        t0 = time.perf_counter()
        if w["bwd"]:
            (O.linear_grads if w["kind"] == "linear" else O.mlp_grads)(d, dO)
        else:
            with torch.no_grad():
                if w["kind"] == "linear":
                    O.linear_scan(*(d[k] for k in LIN))
                else:
                    O.mlp_scan(*(d[k] for k in MLP))
        dt = time.perf_counter() - t0
        best = dt if best is None else min(best, dt)
        reps += 1
    sample = f"B={B} NH={NH} L={w['L']} (full sequence, batch/head slice), fp32, best of {reps}"
    return tokens / best, threads, sample


def forecaster_cpu_reference(w, budget_s=12.0):
    """The forecaster's training-step forward+backward restated on the host cores
    (oracle/ttt_oracle.py forecaster_grads: the reference's ops/ scan and layer code), fp32,
    on a bounded sample: a few windows of the full lookback through all layers."""
    sys.path.insert(0, os.path.join(HERE, "oracle"))
    import synthetic as S
    import ttt_oracle as O
    from forecaster import TTTForecaster

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    B = 2
    cs, lr = w.get("cs", CS), w.get("base_lr", BASE_LR)
    model = TTTForecaster(w["channels"], w["channels"], w["horizon"], w["L"], model_dim=w["NH"] * w["F"],
                          num_heads=w["NH"], num_layers=w["layers"], mini_batch_size=cs, ttt_base_lr=lr,
                          scan_checkpoint_group_size=w["ckpt"], mem_cache_segment_n_mini_batches=w["memo"])
    P = {k: v.detach() for k, v in model.named_parameters()}
    series = S.make_forecast_series(channels=w["channels"], seed=0)
    x, y = S.forecast_windows(series, w["L"], w["horizon"], B, torch.Generator().manual_seed(0))
    lay = model.layers[0]
    prefixes = [f"layers.{i}." for i in range(w["layers"])]
    best, reps = None, 0
    t_end = time.perf_counter() + budget_s
    while reps < 1 or (time.perf_counter() < t_end and reps < 5):
        t0 = time.perf_counter()
        O.forecaster_grads(P, x, y, prefixes, lay.rope_cos, lay.rope_sin, w["horizon"], cs, lr, w["ckpt"],
                           w["memo"])
        dt = time.perf_counter() - t0
        best = dt if best is None else min(best, dt)
        reps += 1
    tokens = B * w["NH"] * w["L"] * w["layers"]
    return tokens / best, threads, f"{B} windows x {w['layers']} layers, full lookback {w['L']}, fp32, fwd+bwd, best of {reps}"


def run_forecaster(args, w, rank, world, local_rank):
    """Training steps of the config-4 forecaster (strong scaling: global batch split over
    the ranks, DDP gradient all-reduce over NCCL)."""
    import _lib
    import synthetic as S
    from forecaster import GraphedTrainStep, TTTForecaster, make_optimizer, train_step

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if w["B"] % world:
        raise SystemExit(f"global batch {w['B']} does not split over {world} ranks")
    b_rank = w["B"] // world
    torch.manual_seed(0)  # identical initial parameters on every rank
    model = TTTForecaster(w["channels"], w["channels"], w["horizon"], w["L"], model_dim=w["NH"] * w["F"],
                          num_heads=w["NH"], num_layers=w["layers"], mini_batch_size=w.get("cs", CS),
                          ttt_base_lr=w.get("base_lr", BASE_LR), scan_checkpoint_group_size=w["ckpt"],
                          mem_cache_segment_n_mini_batches=w["memo"], act_dtype=DT[w["dtype"]]).to(dev)
    net = model
    if world > 1:
        net = torch.nn.parallel.DistributedDataParallel(model, device_ids=[local_rank])
    graphed = world == 1 and not args.no_graph  # one CUDA-graph replay per step on one GPU
    opt = make_optimizer(model, capturable=graphed)
    series = S.make_forecast_series(channels=w["channels"], seed=0)
    gen = torch.Generator().manual_seed(1000 + rank)
    pool = [S.forecast_windows(series, w["L"], w["horizon"], b_rank, gen) for _ in range(4)]
    dev_pool = [(x.to(dev), y.to(dev)) for x, y in pool]

    def barrier():
        if world > 1:
            import torch.distributed as dist

            dist.barrier()

    step_fn = lambda x, y: train_step(net, opt, x, y)  # noqa: E731
    per_step_launches = None
    if graphed:
        n0 = _lib.launch_count()
        step_fn = GraphedTrainStep(net, opt, *dev_pool[0], warmup=args.warmup)
        # library kernels in the captured step (the warm-up steps' launches counted first)
        per_step_launches = _lib.launch_count() - n0
        per_step_launches //= args.warmup + 1
    else:
        for i in range(args.warmup):
            step_fn(*dev_pool[i % 4])
    torch.cuda.synchronize()
    sampler = ClockSampler(smi_index(dev))
    sampler.start()
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    n0 = _lib.launch_count()
    ev0.record(stream)
    for i in range(args.steps):
        step_fn(*dev_pool[i % 4])
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier()
    launches = _lib.launch_count() - n0 if per_step_launches is None else per_step_launches * args.steps
    clocks = sampler.stop()
    ms = ev0.elapsed_time(ev1)
    # dominant kernel (largest share of the step's launch list, profiles/
    # launches_forecaster_config4.md): one layer's F x F scan backward at the per-rank shape
    kern_ms, kern_flops = forecaster_mlp_bwd_ms(w, b_rank, dev)
    # its DRAM traffic from the ncu capture at batch 128 (profiles/mlp_bwd_tc_fxf_config4.md),
    # scaled by the streams (traffic grows in proportion to them)
    kern_traffic = FXF_BWD_TRAFFIC_B128 * b_rank / 128 if w.get("cs", CS) == CS else None
    # end to end: each step's windows copied from pinned host memory, loss read back
    host = [(x.pin_memory(), y.pin_memory()) for x, y in pool]
    xb, yb = torch.empty_like(dev_pool[0][0]), torch.empty_like(dev_pool[0][1])
    loss_host = torch.empty((), dtype=torch.float32).pin_memory()
    torch.cuda.synchronize()
    barrier()  # every rank starts the end-to-end region together (the first all-reduce waits otherwise)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        hx, hy = host[i % 4]
        if graphed:  # straight into the captured step's input buffers
            loss_host.copy_(step_fn(hx, hy), non_blocking=True)
            continue
        xb.copy_(hx, non_blocking=True)
        yb.copy_(hy, non_blocking=True)
        loss_host.copy_(step_fn(xb, yb), non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    ms, e2e_ms = max_over_ranks([ms, e2e_ms], world, dev)
    if rank != 0:
        return
    ms_step = ms / args.steps
    tokens = w["B"] * w["NH"] * w["L"] * w["layers"]  # global, every layer's scan tokens
    hbm, bf16, bf16_sus, src = peaks()
    achieved = kern_flops / (kern_ms / 1e3) / 1e12
    line = {
        "metric": METRIC, "value": tokens / (ms_step / 1e3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": w["dtype"], "data": "synthetic",
        "config": {"workload": args.workload, "global_batch": w["B"], "batch_per_rank": b_rank, "layers": w["layers"],
                   "d_model": w["NH"] * w["F"], "NH": w["NH"], "L": w["L"], "horizon": w["horizon"],
                   "channels": w["channels"], "CS": w.get("cs", CS), "inner": f"F x F ({w['F']})",
                   "base_lr": w.get("base_lr", BASE_LR), "memo_segment_size": w["memo"],
                   "checkpoint_group_size": w["ckpt"], "parallelism": f"dp{world} (DDP, NCCL all-reduce)",
                   "tokens": "B * NH * L per TTT layer, summed over layers",
                   "samples_per_s": w["B"] / (ms_step / 1e3),
                   "cuda_graph": graphed,
                   "l2": "activations larger than L2 (no flush)"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": bf16, "unit": "TFLOP/s",
                     "frac": achieved / bf16, "traffic": kern_traffic,
                     "traffic_source": ("profiles/mlp_bwd_tc_fxf_config4.md (batch 128, scaled)"
                                        if kern_traffic is not None else None),
                     "peak_source": src, "kernel": "mlp_bwd F x F scan backward (one layer)",
                     "kernel_ms": kern_ms, "kernel_flops": kern_flops},
        "e2e": {"value": tokens / (e2e_ms / args.steps / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": (xb.numel() * xb.element_size() + yb.numel() * yb.element_size()),
                "d2h_bytes_per_step": 4, "ms_per_step": e2e_ms / args.steps},
        "gpu_launches": launches,
        "clocks": clocks,
    }
    if world == 1 and not args.no_cpu_baseline:
        v, cores, sample = forecaster_cpu_reference(w)
        line["cpu_baseline"] = {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample}
    print(json.dumps(line), flush=True)


# DRAM bytes (read + write) of one F x F scan-backward launch at batch 128 (ncu capture in
# profiles/mlp_bwd_tc_fxf_config4.md)
FXF_BWD_TRAFFIC_B128 = 286.697984e6 + 73.438464e6


def forecaster_mlp_bwd_ms(w, b_rank, dev):
    """Device time of one layer's scan backward at the per-rank shape, averaged over
    back-to-back launches (the stored-pre-activation tensor-core path the config-4 layer
    takes; the general kernel for main.py's CS 64, head_dim 32), and its useful FLOPs:
    38 F FF + 12 CS FF + 12 CS F per token (algorithmic())."""
    import _core
    import synthetic as S

    cs = w.get("cs", CS)
    NC, F, FF = w["L"] // cs, w["F"], w["FF"]
    dt = DT[w["dtype"]]
    d = S.make_mlp_inputs(b_rank, w["NH"], NC, cs, F, FF, dtype=dt, device=dev, seed=5)
    dO = S.make_upstream((b_rank, w["NH"], NC, cs, F), device=dev, seed=6, dtype=dt)
    _, last, ck, _, zs = _core.mlp_forward(d["ln_w"], d["ln_b"], d["W1"], d["b1"], d["W2"], d["b2"], d["XQ"], d["XV"],
                                           d["XK"], d["eta"], min(w["ckpt"], NC), w["memo"], for_backward=True)
    stream = torch.cuda.current_stream(dev)

    def bwd():
        _core.mlp_backward(d["ln_w"], d["ln_b"], ck, d["XQ"], d["XV"], d["XK"], d["eta"], dO, min(w["ckpt"], NC),
                           saved=zs, W1_last=last[0], W2_last=last[2])

    bwd()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(5):
        bwd()
    e1.record(stream)
    torch.cuda.synchronize()
    flops = (38 * F * FF + 12 * cs * FF + 12 * cs * F) * b_rank * w["NH"] * w["L"]
    return e0.elapsed_time(e1) / 5, flops


def cpu_full_shape(w, steps, warmup):
    """The reference's ops/ path restated on the host cores (oracle/ttt_oracle.py, fp32) at
    the workload's FULL shape: every step runs all B * NH streams over the whole sequence,
    in chunks of 4 streams (batched matmuls over all streams at once run several times
    slower on the host, cache-bound). Warm-up steps run one chunk each. Returns (tokens/s
    over the timed steps, threads, sample description)."""
    sys.path.insert(0, os.path.join(HERE, "oracle"))
    import synthetic as S
    import ttt_oracle as O

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    NC = w["L"] // CS
    mk = S.make_linear_inputs if w["kind"] == "linear" else S.make_mlp_inputs
    kw = {} if w["kind"] == "linear" else {"FF": w["FF"]}
    d = mk(w["B"], w["NH"], NC, CS, w["F"], seed=0, **kw)
    names = LIN if w["kind"] == "linear" else MLP
    scan = O.linear_scan if w["kind"] == "linear" else O.mlp_scan
    chunks = []
    for b in range(w["B"]):
        for h0 in range(0, w["NH"], 4):
            h1 = min(h0 + 4, w["NH"])
            chunks.append({k: (v[h0:h1] if k in ("ln_w", "ln_b") else v[b:b + 1, h0:h1]) for k, v in d.items()})
    extra = () if w["kind"] == "linear" else (w["ckpt"], memo_of(w))

    def one(c):
        with torch.no_grad():
            scan(*(c[k] for k in names), *extra)

    for _ in range(warmup):
        one(chunks[0])
    t0 = time.perf_counter()
    for _ in range(steps):
        for c in chunks:
            one(c)
    dt = time.perf_counter() - t0
    tokens = w["B"] * w["NH"] * w["L"] * steps
    sample = (f"full shape B={w['B']} NH={w['NH']} L={w['L']}, {steps} step(s), all streams in chunks of 4, "
              f"fp32, forward")
    return tokens / dt, threads, sample


def run_reference(args, w, rank, world):
    """The reference arm: rank 0 alone times the CPU port of the reference's ops/ path on the
    host cores, on this arm's workload and config; other ranks exit without work."""
    if rank != 0:
        return
    config = {"workload": args.workload, **{k: v for k, v in w.items() if k in ("B", "NH", "L", "F", "FF")}}
    if w["kind"] in ("linear", "mlp") and not w["bwd"]:
        value, cores, sample = cpu_full_shape(w, args.steps, args.warmup)
        config = ours_config(args, w, 1)
    elif w["kind"] == "forecaster":
        value, cores, sample = forecaster_cpu_reference(w)
    else:
        value, cores, sample = cpu_reference(w)
        config["shape_run"] = sample
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
        "scaling": "strong" if w["kind"] == "forecaster" else "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": config,
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def ours_config(args, w, world, sharded=False):
    """The `config` object of a line (the reference arm reports the same one)."""
    par = (f"batch split over {world} GPU(s) (strong scaling), no collective" if sharded
           else f"streams sharded over {world} GPU(s), no collective")
    return {"workload": args.workload, "B_per_rank": w["B"], "NH": w["NH"],
            "L": w["L"], "F": w["F"], "FF": w["FF"], "CS": CS, "checkpoint_group_size": w["ckpt"],
            "memo_segment_size": memo_of(w) if w["kind"] == "mlp" else w["memo"],
            "global_batch": w["B"] * (1 if sharded else world), "parallelism": par,
            "l2": "inputs larger than L2 (no flush)"}


def measure(args, w, d, dO, dev, rank, world, global_tokens, with_cpu):
    """Device-timed steps of workload w on this rank's inputs (barrier + synchronize around
    the region, max over ranks), the dominant kernel's back-to-back launch time and the
    end-to-end leg. Returns the record on rank 0 (None elsewhere): step time, tokens/s of the
    whole job (global_tokens per step), roofline, e2e, launches, clocks, CPU baseline."""
    import torch.distributed as dist

    def barrier():
        if world > 1:
            dist.barrier()

    tokens_rank = w["B"] * w["NH"] * w["L"]
    for _ in range(args.warmup):
        kernel_step(w, d, dO)
    torch.cuda.synchronize()
    sampler = ClockSampler(smi_index(dev))
    sampler.start()
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    ev0.record(stream)
    launches = 0
    for _ in range(args.steps):
        launches += kernel_step(w, d, dO)
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    ms = ev0.elapsed_time(ev1)
    kern_ms, kname = kernel_durations(w, d, dO, args.steps)
    e2e_ms, h2d, d2h = e2e_time(w, d, dO, dev, args)
    ms, e2e_ms, kern_ms = max_over_ranks([ms, e2e_ms, kern_ms], world, dev)
    if rank != 0:
        return None
    ms_step = ms / args.steps
    hbm, bf16, bf16_sus, src = peaks()
    alg = algorithmic(w)
    dom = "bwd" if w["bwd"] else "fwd"  # dominant kernel: the backward when there is one
    dom_bytes, dom_flops = alg[dom]
    if w["kind"] in ("mlp", "memo"):
        achieved = dom_flops * tokens_rank / (kern_ms / 1e3) / 1e12
        roof = {"bound": "tensor", "achieved": achieved, "peak": bf16, "unit": "TFLOP/s", "frac": achieved / bf16}
    else:
        achieved = dom_bytes * tokens_rank / (kern_ms / 1e3) / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm}
    traffic = NCU_TRAFFIC.get((w.get("name", args.workload), kname))
    roof.update({
        "traffic": traffic[0] * (tokens_rank / traffic[1]) if traffic else None,
        "traffic_source": traffic[2] if traffic else None,
        "peak_source": src,
        "kernel": kname,
        "kernel_ms": kern_ms,
        "kernel_timing": "back-to-back launches between CUDA events, average (max over ranks)",
        "algorithmic_bytes_per_token": dom_bytes,
        "algorithmic_flops_per_token": dom_flops,
    })
    step_bytes = alg["fwd"][0] + (alg["bwd"][0] if w["bwd"] else 0)
    step_flops = alg["fwd"][1] + (alg["bwd"][1] if w["bwd"] else 0)
    roof["hbm_roofline_tokens_per_s"] = hbm * 1e9 / step_bytes
    roof["hbm_frac_of_step"] = (tokens_rank / (ms_step / 1e3)) / roof["hbm_roofline_tokens_per_s"]
    roof["tensor_roofline_tokens_per_s"] = bf16 * 1e12 / step_flops
    roof["tensor_frac_of_step"] = (tokens_rank / (ms_step / 1e3)) / roof["tensor_roofline_tokens_per_s"]
    rec = {
        "value": global_tokens / (ms_step / 1e3), "unit": "tokens/s", "ms_per_step": ms_step,
        "roofline": roof,
        "e2e": {"value": global_tokens / (e2e_ms / args.steps / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world,
                "ms_per_step": e2e_ms / args.steps},
        "gpu_launches": launches,
        "clocks": clocks,
    }
    if with_cpu:
        v, cores, sample = cpu_reference(w)
        rec["cpu_baseline"] = {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample}
    return rec


FWDBWD_RECORDS = (
    ("mlp_fwdbwd_c3", "fwdbwd", "TTT-MLP fwd+bwd tokens/s (B*H*L), config 3 global batch split over the GPUs"),
    ("linear_fwdbwd_c2", "fwdbwd_linear",
     "TTT-Linear fwd+bwd tokens/s (B*H*L), config 2 global batch split over the GPUs"),
)


def run_fwdbwd_sharded(args, rank, world, dev, workload, metric):
    """A training config (config 3: TTT-MLP, B64 NH16 L8192; config 2: TTT-Linear, B32 NH8
    L4096; forward+backward) as one global batch split over the ranks by batch
    (sharding.shard), strong scaling. Every rank builds the same seeded global inputs on its
    device, keeps its slice and frees the rest."""
    import sharding

    w = dict(WORKLOADS[workload], name=workload)
    Bg = w["B"]
    if Bg % world:
        raise SystemExit(f"{workload} batch {Bg} does not split over {world} ranks")
    g, gO = make_inputs(w, dev, seed=0)
    d = sharding.shard(g, rank, world)
    b0, b1 = sharding.batch_range(Bg, rank, world)
    dO = gO[b0:b1].contiguous()
    del g, gO
    torch.cuda.empty_cache()
    wr = dict(w, B=b1 - b0)
    rec = measure(args, wr, d, dO, dev, rank, world, Bg * w["NH"] * w["L"],
                  with_cpu=(world == 1 and not args.no_cpu_baseline))
    del d, dO
    torch.cuda.empty_cache()
    if rec is None:
        return None
    rec["config"] = ours_config(args, dict(w, B=Bg // world), world, sharded=True)
    rec["config"]["workload"] = workload
    rec["config"]["global_batch"] = Bg
    rec["scaling"] = "strong"
    rec["metric"] = metric
    return rec


def run_ours(args, w, rank, world, local_rank):
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    d, dO = make_inputs(w, dev, seed=rank)
    tokens_rank = w["B"] * w["NH"] * w["L"]
    rec = measure(args, w, d, dO, dev, rank, world, world * tokens_rank, with_cpu=(world == 1 and not args.no_cpu_baseline))
    del d, dO
    torch.cuda.empty_cache()
    records = {}
    if args.workload == "mlp_fwd_c1" and not args.no_fwdbwd:
        for workload, key, metric in FWDBWD_RECORDS:
            records[key] = run_fwdbwd_sharded(args, rank, world, dev, workload, metric)
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": rec["value"], "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": rec["ms_per_step"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": w["dtype"], "data": "synthetic",
        "config": ours_config(args, w, world),
    }
    line.update({k: v for k, v in rec.items() if k not in ("value", "unit", "ms_per_step")})
    line.update(records)
    print(json.dumps(line), flush=True)


def max_over_ranks(times, world, device):
    """Each timing is the max over ranks (the slowest rank bounds the job)."""
    if world == 1:
        return list(times)
    import torch.distributed as dist

    t = torch.tensor(list(times), device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(x) for x in t]


def weak_scaling_value(world, tokens_per_rank, ms_per_step):
    """Whole-job tokens/s: every rank processes its own batch of tokens_per_rank."""
    return world * tokens_per_rank / (ms_per_step / 1e3)


def dominant_launch(w, d, dO):
    """A closure that enqueues one call of the dominant kernel's entry point (the backward
    when the workload has one), with every input it reads prepared beforehand (the forward
    it follows has run), and that kernel's name."""
    import _core

    if w["kind"] == "prologue":
        from prologue import concat_projections

        B, L, NH, F = w["B"], w["L"], w["NH"], w["F"]
        Wcat, bcat, _, _ = concat_projections(*(d[k] for k in PRO[1:11]))
        P = torch.addmm(bcat, d["hidden"].reshape(B * L, -1), Wcat.t())
        scale = BASE_LR / (F * CS)
        return (lambda: _core.prologue_backward(P, B, L, NH, F, CS, d["ln_w"], d["ln_b"], d["freqs_cos"],
                                                d["freqs_sin"], scale, *(dO[k] for k in PRO_OUTS))), "prologue_bwd"
    if w["kind"] == "epilogue":
        Y = _core.post_norm_forward(d["XQW"], d["pn_w"], d["pn_b"], POST_NORM_EPS)
        d2 = dO.reshape(Y.shape)
        dY = torch.mm(d2, d["wo_w"])
        return (lambda: _core.post_norm_backward(d["XQW"], d["pn_w"], d["pn_b"], POST_NORM_EPS, dY, d2)), \
            "post_norm_bwd"
    if w["kind"] == "memo":
        _, scratch = _core.memo_mix_forward(*(d[k] for k in MEMO), w["memo"], return_scratch=True)
        return (lambda: _core.memo_mix_backward(*(d[k] for k in MEMO), w["memo"], dO, scratch=scratch)), \
            "memo_bwd (mix + dXK launches)"
    if w["kind"] == "linear":
        if w["bwd"]:
            _, Wl, bl, Wc, bc, Z = _core.linear_forward(*(d[k] for k in LIN), w["ckpt"])
            return (lambda: _core.linear_backward(d["ln_w"], d["ln_b"], Wc, bc, d["XQ"], d["XV"], d["XK"], d["eta"],
                                                  dO, w["ckpt"], Z=Z, W_last=Wl, b_last=bl)), "linear_bwd"
        return (lambda: _core.linear_forward(*(d[k] for k in LIN), w["ckpt"], for_backward=False)), "linear_fwd"
    if w["bwd"]:
        _, last, ck, _, zs = _core.mlp_forward(*(d[k] for k in MLP), w["ckpt"], memo_of(w))
        return (lambda: _core.mlp_backward(d["ln_w"], d["ln_b"], ck, d["XQ"], d["XV"], d["XK"], d["eta"], dO,
                                           w["ckpt"], saved=zs, W1_last=last[0], W2_last=last[2])), "mlp_bwd"
    return (lambda: _core.mlp_forward(*(d[k] for k in MLP), w["ckpt"], memo_of(w), for_backward=False)), "mlp_fwd"


def kernel_durations(w, d, dO, steps):
    """Average device time of one launch of the dominant kernel: n calls enqueued back to
    back between two CUDA events on their stream, so the host work of each call (output
    allocation, tensor-map encoding) overlaps the previous launch and the GPU never idles
    between them. Returns (ms per launch, kernel name)."""
    launch, name = dominant_launch(w, d, dO)
    stream = torch.cuda.current_stream()
    n = max(3, min(steps, 10))
    launch()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(n):
        launch()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / n, name


def e2e_time(w, d, dO, dev, args):
    """End-to-end steps through the public API with host buffers. Every step copies all of
    its inputs from pinned host memory to the device, runs api_compute and reads its result
    back to pinned host memory, all inside the timed region. Steps are pipelined as a data
    loader would feed them: uploads on one stream, readbacks on another, two device buffer
    sets, so step k+1's upload and step k-1's readback overlap step k's compute (a buffer
    set is refilled only after the compute two steps back has finished with it). Returns
    (ms for args.steps steps, H2D bytes per step, D2H bytes per step)."""
    host = {k: v.detach().cpu().pin_memory() for k, v in d.items()}
    if isinstance(dO, dict):
        host.update({"d_" + k: v.cpu().pin_memory() for k, v in dO.items()})
    elif dO is not None:
        host["dO"] = dO.cpu().pin_memory()
    bufs = [{k: torch.empty_like(v, device=dev) for k, v in host.items()} for _ in range(2)]
    res_like = d[RESULT_KEY.get(w["kind"], "XQ")]
    out_host = [torch.empty(res_like.shape, dtype=res_like.dtype).pin_memory() for _ in range(2)]
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = out_host[0].numel() * out_host[0].element_size()
    comp = torch.cuda.current_stream(dev)
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def run(n):
        loaded = [torch.cuda.Event(), torch.cuda.Event()]
        done = [torch.cuda.Event(), torch.cuda.Event()]
        up.wait_stream(comp)
        down.wait_stream(comp)
        for i in range(n):
            b = i % 2
            with torch.cuda.stream(up):
                if i >= 2:
                    up.wait_event(done[b])  # compute of step i - 2 is done with buffer set b
                for k, t in host.items():
                    bufs[b][k].copy_(t, non_blocking=True)
                loaded[b].record(up)
            comp.wait_event(loaded[b])
            res = api_compute(w, bufs[b])
            done[b].record(comp)
            with torch.cuda.stream(down):
                down.wait_event(done[b])
                res.record_stream(down)  # keep the result allocated until its readback ran
                out_host[b].copy_(res, non_blocking=True)
        comp.wait_stream(up)
        comp.wait_stream(down)

    run(max(2, min(args.warmup, 2)))
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    run(args.steps)
    e1.record(comp)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1), h2d, d2h


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="mlp_fwd_c1")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true",
                    help="forecaster workloads on one GPU: eager steps instead of one CUDA-graph replay per step")
    ap.add_argument("--no-fwdbwd", action="store_true",
                    help="skip the config-3 forward+backward record of the default workload")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the workload's per-rank batch (smaller cases for profiling)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    w = dict(WORKLOADS[args.workload])
    if args.batch is not None:
        if args.batch <= 0:
            raise SystemExit("--batch must be positive")
        w["B"] = args.batch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, w, rank, world)
        return
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        if w["kind"] == "forecaster":
            run_forecaster(args, w, rank, world, local_rank)
        else:
            run_ours(args, w, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
