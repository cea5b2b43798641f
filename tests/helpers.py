"""Shared test helpers: golden loading, oracle runs and tolerance checks."""

from __future__ import annotations

import os

import numpy as np
import torch

import ttt_oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

# Parity bars of the north star: relative L2 error.
TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2, torch.float16: 2e-2}


def load_golden(name):
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    inp = {k[3:]: torch.from_numpy(z[k]) for k in z.files if k.startswith("in_")}
    extra = {k: torch.from_numpy(z[k]) for k in z.files if not k.startswith("in_")}
    return inp, extra


def to_dev(d, device, act_dtype=None):
    """Move an input dict to device; activations (XQ/XK/XV/eta) cast to act_dtype."""
    out = {}
    for k, v in d.items():
        v = v.to(device)
        if act_dtype is not None and k in ("XQ", "XK", "XV", "eta"):
            v = v.to(act_dtype)
        out[k] = v
    return out


def oracle_inputs(d):
    """float64 CPU copy of the (possibly low-precision-rounded) inputs the kernel sees."""
    return {k: v.detach().to("cpu", torch.float64) for k, v in d.items()}


def assert_close(name, got, ref, tol):
    err = O.rel_l2(got.detach().to("cpu", torch.float64), ref.detach().to("cpu", torch.float64))
    assert err <= tol, f"{name}: relative L2 error {err:.3e} > {tol:.1e}"
    return err
