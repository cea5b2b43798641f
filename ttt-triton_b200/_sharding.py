"""Head-sharded (tensor-parallel) entry support shared by the autograd wrappers.

The reference wraps its cores in torch's ``local_map`` so that DTensor inputs sharded on
the head dimension run the kernel on their local shard (linear_triton.py:267-357,
mlp_triton.py:353-463). The same placements are declared here; with plain tensors
``local_map`` passes them through unchanged.
"""

from __future__ import annotations

try:  # torch >= 2.5 public location
    from torch.distributed.tensor import Shard
    from torch.distributed.tensor.experimental import local_map
except ImportError:  # pragma: no cover - older torch
    from torch.distributed._tensor import Shard
    from torch.distributed._tensor.experimental import local_map

HEAD = [Shard(1)]  # activations, states, per-(b,h) tensors: heads on dim 1
LN = [Shard(0)]  # ttt_norm_weight / ttt_norm_bias [NH, F]: heads on dim 0

__all__ = ["local_map", "HEAD", "LN"]
