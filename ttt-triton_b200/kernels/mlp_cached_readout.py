"""Drop-in for ``kernels.mlp_cached_readout.mlp_cached_readout_triton`` (kernels/mlp_cached_readout.py:112-143).

    out = mlp_cached_readout_triton(XQ_seg [B,NH,NCseg,CS,F], W1 [B,NH,F,FF], b1 [B,NH,1,FF],
                                    W2 [B,NH,FF,F], b2 [B,NH,1,F], ln_w [NH,F], ln_b [NH,F])

returns fp32 ``XQ_seg + LN(gelu(XQ_seg W1 + b1) W2 + b2)`` (LayerNorm eps 1e-6, the
kernel's constant). The state tensors may be the non-contiguous memo slices
``W1_memo[:, :, j]`` the layer passes (ttt_layer.py:543-552): their batch/head strides go
to the kernel. Every (b, h) is read and written at its own offset.
"""

from __future__ import annotations

import _core


def mlp_cached_readout_triton(XQ_seg, W1, b1, W2, b2, ln_w, ln_b):
    return _core.mlp_cached_readout(XQ_seg, W1, b1, W2, b2, ln_w, ln_b)
