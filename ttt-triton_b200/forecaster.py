"""TTT-MLP forecaster on the sm_100a kernels: the reference's TTTForecaster (forecast.py:
79-99) with a stack of TTT-MLP layers (ttt_layer.py:59-357, 423-565) whose every stage runs
on this library.

A layer is the reference's TTTMLP (TTTBase parameters and an F x F inner MLP) with its
forward (ttt_layer.py:337-357) as four calls:

    inputs = prologue.ttt_prologue(...)                # process_input, :261-330
    XQW, *memo = TritonMLP.apply(...)                  # the dual-form scan, :467-488
    XQW = mlp_memo_mix(XQW, ..., memo_segment_size)    # memo mixing, :503-559
    out = epilogue.post_norm_wo(XQW, ...)              # permute + post_norm + wo, :349-350, 563-564

Parameter names match the reference's modules, so its state dicts load
(``load_reference_state_dict``). Activations run in ``act_dtype`` (bf16 by default, the
16-bit training the reference gets from autocast); parameters and the inner states stay
fp32.

``train_step`` is one optimisation step of main.py:73-100 (AdamW, MSE, gradient clipping at
1.0); under torch.distributed the model is wrapped in DistributedDataParallel and the
outer-parameter gradients are averaged by NCCL all-reduce over NVLink.
"""

from __future__ import annotations

import torch
import torch.nn.functional as Fn
from torch import nn

import epilogue
import prologue
from kernels.mlp_memo_mix import mlp_memo_mix
from mlp_triton import TritonMLP


def rope_table_3d(head_dim, height, width, frames, theta=10000.0):
    """fp32 (cos, sin) [frames * height * width, head_dim / 2] of the reference's rotary
    frequencies (utils.py:24-71, precompute_freqs_cis_3d): head_dim / 4 dimensions rotate
    with the frame index, 3 * head_dim / 8 each with the row and the column (rows and
    columns are position 0 for a 1 x 1 latent, so those pairs do not rotate)."""
    dim_t, dim_h = head_dim // 4, head_dim // 8 * 3
    dim_w = dim_h

    def freqs(dim, n):
        inv = 1.0 / (theta ** (torch.arange(0, dim, 2)[: dim // 2].float() / dim))
        return torch.arange(n, dtype=torch.float32)[:, None] * inv[None, :]

    ft, fh, fw = freqs(dim_t, frames), freqs(dim_h, height), freqs(dim_w, width)
    ang = torch.cat([
        ft[:, None, None, :].expand(frames, height, width, ft.shape[-1]),
        fh[None, :, None, :].expand(frames, height, width, fh.shape[-1]),
        fw[None, None, :, :].expand(frames, height, width, fw.shape[-1]),
    ], dim=-1).reshape(frames * height * width, -1)
    return torch.cos(ang), torch.sin(ang)


_ONES = {}


def _ones(n, like):
    key = (n, like.device, like.dtype)
    if key not in _ONES:
        _ONES[key] = torch.ones(n, device=like.device, dtype=like.dtype)
    return _ONES[key]


class BatchCopies(torch.autograd.Function):
    """p -> B contiguous copies [B, *p.shape], the per-sequence initial inner states of
    ttt_layer.py:462-465 (``torch.tile(p.unsqueeze(0), (B, 1, ...))``). The backward sums
    the B gradient copies with one matrix-vector product (a strided reduction over the
    leading dimension is several times slower for these shapes)."""

    @staticmethod
    def forward(ctx, p, B):
        ctx.B = B
        return p.unsqueeze(0).expand(B, *p.shape).contiguous()

    @staticmethod
    def backward(ctx, g):
        B = ctx.B
        g2 = g.reshape(B, -1)
        return torch.mv(g2.t(), _ones(B, g2)).reshape(g.shape[1:]), None


class TTTMLPLayer(nn.Module):
    """ttt_layer.TTTMLP with use_kernel=True on this library (no tensor parallelism)."""

    def __init__(self, model_dim, num_heads, mini_batch_size, seq_len, ttt_base_lr=0.1,
                 scan_checkpoint_group_size=16, mem_cache_segment_n_mini_batches=2, rope_theta=10000.0,
                 latent_height=1, latent_width=1, act_dtype=torch.bfloat16):
        super().__init__()
        if model_dim % num_heads:
            raise ValueError("model_dim must be a multiple of num_heads")
        self.width, self.num_heads = model_dim, num_heads
        self.head_dim = model_dim // num_heads
        self.mini_batch_size = mini_batch_size
        self.ttt_base_lr = ttt_base_lr
        self.scan_checkpoint_group_size = scan_checkpoint_group_size
        self.mem_cache_segment_n_mini_batches = mem_cache_segment_n_mini_batches
        self.act_dtype = act_dtype
        self.tp_mesh = None
        W, NH, F = model_dim, num_heads, self.head_dim
        # TTTBase._init_qkvo_proj / _init_ttt_lr_gate / _init_ttt_ln (ttt_layer.py:91-119)
        self.wq, self.wk, self.wv, self.wo, self.wu = (nn.Linear(W, W) for _ in range(5))
        self.learnable_ttt_lr_weight = nn.Parameter(torch.normal(0, 0.02, size=(NH, 1, W)))
        self.learnable_ttt_lr_bias = nn.Parameter(torch.zeros(NH, 1))
        self.ttt_norm_weight = nn.Parameter(torch.ones(NH, F))
        self.ttt_norm_bias = nn.Parameter(torch.zeros(NH, F))
        self.post_norm = nn.LayerNorm(W, eps=1e-6)
        # TTTMLP inner MLP (ttt_layer.py:427-430): F x F, GELU
        self.W1 = nn.Parameter(torch.normal(0, 0.02, size=(NH, F, F)))
        self.b1 = nn.Parameter(torch.zeros(NH, 1, F))
        self.W2 = nn.Parameter(torch.normal(0, 0.02, size=(NH, F, F)))
        self.b2 = nn.Parameter(torch.zeros(NH, 1, F))
        cos, sin = rope_table_3d(F, latent_height, latent_width, seq_len, rope_theta)
        self.register_buffer("rope_cos", cos, persistent=False)
        self.register_buffer("rope_sin", sin, persistent=False)

    def forward(self, hidden_states):
        B, L, _ = hidden_states.shape
        if L % self.mini_batch_size:
            raise ValueError("Sequence len must be multiple of mini batch size.")
        x = hidden_states.to(self.act_dtype)
        inputs = prologue.process_input(self, x, (self.rope_cos, self.rope_sin))
        NC = inputs["XV"].shape[2]
        ckpt = min(max(self.scan_checkpoint_group_size, 1), NC)
        memo = self.mem_cache_segment_n_mini_batches
        XQW, W1_memo, b1_memo, W2_memo, b2_memo = TritonMLP.apply(
            self.ttt_norm_weight, self.ttt_norm_bias, BatchCopies.apply(self.W1, B), BatchCopies.apply(self.b1, B),
            BatchCopies.apply(self.W2, B), BatchCopies.apply(self.b2, B), inputs["XQ"], inputs["XV"], inputs["XK"],
            inputs["eta"], ckpt, memo)
        XQW = mlp_memo_mix(XQW, inputs["XQ"], inputs["XK"], inputs["XU"], W1_memo, b1_memo, W2_memo, b2_memo,
                           self.ttt_norm_weight, self.ttt_norm_bias, memo)
        return epilogue.output_epilogue(self, XQW)


def linear_act(x, weight, bias, dt):
    """nn.Linear in the activation dtype dt (what the reference's autocast runs), with the
    input width padded to a multiple of 8 so that the library GEMMs take their aligned
    tensor-core paths (the 7-channel input projection and its weight gradient otherwise fall
    back to unaligned fp32 kernels). The first padding column carries the bias: the input
    gets a column of ones and the weight the bias as that column, so the bias gradient comes
    out of the weight-gradient GEMM instead of a separate reduction over all B * L rows."""
    k = x.shape[-1]
    pad = -k % 8
    if not pad:
        return Fn.linear(x.to(dt), weight.to(dt), bias.to(dt))
    x = Fn.pad(x, (0, 1), value=1.0)
    cols = [weight, bias[:, None]]
    if pad > 1:
        x = Fn.pad(x, (0, pad - 1))
        cols.append(weight.new_zeros(weight.shape[0], pad - 1))
    return Fn.linear(x.to(dt), torch.cat(cols, 1).to(dt))


class TTTForecaster(nn.Module):
    """forecast.TTTForecaster (in_proj -> TTT layers -> head on the last position) with
    num_layers stacked TTT-MLP layers."""

    def __init__(self, d_in, d_out, pred_len, seq_len, model_dim=256, num_heads=4, num_layers=4,
                 mini_batch_size=16, ttt_base_lr=0.1, scan_checkpoint_group_size=16,
                 mem_cache_segment_n_mini_batches=2, act_dtype=torch.bfloat16):
        super().__init__()
        self.pred_len, self.d_out = pred_len, d_out
        self.act_dtype = act_dtype
        self.in_proj = nn.Linear(d_in, model_dim)
        self.layers = nn.ModuleList(
            TTTMLPLayer(model_dim, num_heads, mini_batch_size, seq_len, ttt_base_lr, scan_checkpoint_group_size,
                        mem_cache_segment_n_mini_batches, act_dtype=act_dtype) for _ in range(num_layers))
        self.head = nn.Linear(model_dim, pred_len * d_out)

    def forward(self, seq_x):
        h = linear_act(seq_x, self.in_proj.weight, self.in_proj.bias, self.act_dtype)
        for layer in self.layers:
            h = layer(h)
        out = self.head(h[:, -1].to(self.head.weight.dtype))
        return out.view(seq_x.size(0), self.pred_len, self.d_out)


def load_reference_state_dict(model, state_dict):
    """Load a reference TTTForecaster state dict (one TTT layer under ``ttt.ttt.``) into
    layer 0 of this model; in_proj and head map by name."""
    mapped = {}
    for k, v in state_dict.items():
        if k.startswith("ttt.ttt."):
            mapped["layers.0." + k[len("ttt.ttt."):]] = v
        elif k.startswith("ttt."):
            continue  # the wrapper's buffers (freqs_cis) are rebuilt here
        else:
            mapped[k] = v
    missing, unexpected = model.load_state_dict(mapped, strict=False)
    missing = [k for k in missing if not k.startswith("layers.") or k.startswith("layers.0.")]
    if missing or unexpected:
        raise KeyError(f"state dict mismatch: missing {missing}, unexpected {unexpected}")


def make_optimizer(model, lr=1e-3, weight_decay=1e-2, capturable=False):
    """AdamW as main.py:68 (the fused multi-tensor update on CUDA). capturable keeps the step
    counts on the device, as a CUDA-graph-captured step (GraphedTrainStep) needs."""
    fused = all(p.is_cuda for p in model.parameters())
    return torch.optim.AdamW(model.parameters(), lr=lr, weight_decay=weight_decay, fused=fused,
                             capturable=capturable and fused)


def train_step(model, optimizer, x, y, clip=1.0):
    """One step of main.py:73-100: MSE on the forecast, backward (gradient all-reduce when the
    model is DistributedDataParallel), clipping at `clip`, AdamW. Returns the loss tensor
    (not synchronised)."""
    optimizer.zero_grad(set_to_none=True)
    pred = model(x)
    loss = Fn.mse_loss(pred.float(), y.float())
    loss.backward()
    if clip is not None:
        torch.nn.utils.clip_grad_norm_(model.parameters(), clip)
    optimizer.step()
    return loss.detach()


class GraphedTrainStep:
    """train_step captured once in a CUDA graph and replayed: one graph launch per step
    instead of the step's ~80-400 kernel launches from Python, for a single-GPU model whose
    step is launch-bound (small batches, short sequences). The optimizer must be made with
    make_optimizer(..., capturable=True). Construction runs `warmup` ordinary training steps
    on (x, y) on a side stream (the model trains on them) and then captures one step;
    calling the object copies a batch into the captured input buffers, replays the graph and
    returns the loss tensor of that step (not synchronised). The batch shape is fixed at
    construction. Not for DistributedDataParallel models (their all-reduce is not captured
    here)."""

    def __init__(self, model, optimizer, x, y, clip=1.0, warmup=3):
        if isinstance(model, nn.parallel.DistributedDataParallel):
            raise ValueError("GraphedTrainStep captures single-GPU steps; use train_step with DDP")
        self.x = x.detach().clone()
        self.y = y.detach().clone()
        side = torch.cuda.Stream(device=self.x.device)
        side.wait_stream(torch.cuda.current_stream(self.x.device))
        with torch.cuda.stream(side):  # allocator pools, optimizer state, one-time set-up
            for _ in range(warmup):
                train_step(model, optimizer, self.x, self.y, clip)
        torch.cuda.current_stream(self.x.device).wait_stream(side)
        optimizer.zero_grad(set_to_none=True)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.loss = train_step(model, optimizer, self.x, self.y, clip)

    def __call__(self, x, y):
        self.x.copy_(x, non_blocking=True)
        self.y.copy_(y, non_blocking=True)
        self.graph.replay()
        return self.loss


def tokens_per_step(batch, seq_len, num_heads, num_layers):
    """TTT tokens (b, h, t) one step runs through the scan: every layer's B * NH * L."""
    return batch * num_heads * seq_len * num_layers


__all__ = ["BatchCopies", "linear_act", "TTTMLPLayer", "TTTForecaster", "rope_table_3d", "load_reference_state_dict", "make_optimizer",
           "train_step", "GraphedTrainStep", "tokens_per_step"]
