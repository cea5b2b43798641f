"""ctypes binding of libttt_b200.so (the C ABI declared in include/ttt_b200.h).

The library must exist: there is no fallback path. Import fails with a clear message
when it has not been built (``python ttt-triton_b200/build.py``), and every call checks
that its tensors live on a CUDA device.
"""

from __future__ import annotations

import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
# TTT_B200_LIB names another build of the same ABI in this directory (the timeline build,
# libttt_b200_stamps.so, of build.py --phase-stamps)
LIB_PATH = os.path.join(_HERE, os.environ.get("TTT_B200_LIB", "libttt_b200.so"))

DTYPE_CODES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}

_P = ctypes.c_void_p
_I = ctypes.c_int
_Z = ctypes.c_size_t
_L = ctypes.c_longlong

_SIGNATURES = {
    "ttt_abi_version": ([], _I),
    "ttt_last_error": ([], ctypes.c_char_p),
    "ttt_linear_fwd": ([_I] * 6 + [_P, _P, _I, _P, _P, _P, _I, _P, _I, _P, _I, _P, _I, _P, _I, _P, _P, _P, _P, _P, _P], _I),
    "ttt_linear_bwd_scratch_bytes": ([_I] * 6, _Z),
    "ttt_linear_bwd": (
        [_I] * 6
        + [_P, _P, _I, _P, _P, _P, _I, _P, _I, _P, _I, _P, _I, _P, _I]
        + [_P, _P, _P]
        + [_P, _P, _P, _P, _P, _P, _P, _P, _I, _P, _Z, _P],
        _I,
    ),
    "ttt_linear_bwd_noalloc": (
        [_I] * 6
        + [_P, _P, _I, _P, _P, _P, _I, _P, _I, _P, _I, _P, _I, _P, _I]
        + [_P, _P, _P, _P, _P, _P, _P, _P, _I, _P],
        _I,
    ),
    "ttt_mlp_fwd": (
        [_I] * 8
        + [_P, _P, _I, _P, _P, _P, _P, _P, _I, _P, _I, _P, _I, _P, _I, _P, _I]
        + [_P] * 12
        + [_P] * 4
        + [_P],
        _I,
    ),
    "ttt_mlp_bwd_scratch_bytes": ([_I] * 7, _Z),
    "ttt_mlp_bwd": (
        [_I] * 7
        + [_P, _P, _I, _P, _P, _P, _P, _P, _I, _P, _I, _P, _I, _P, _I, _P, _I]
        + [_P] * 6
        + [_P] * 10
        + [_I, _P, _Z, _P],
        _I,
    ),
    "ttt_device_status": ([_P], _I),
    "ttt_test_hold_first_stage": ([_I, ctypes.c_ulonglong], _I),
    "ttt_kernel_launches": ([], ctypes.c_ulonglong),
    "ttt_set_forward_schedule": ([_I, _I], _I),
    "ttt_mlp_fwd_schedule_plan": ([_I, _I, _I, _I, _P, _P, _I, _P], _I),
    "ttt_memo_mix_scratch_bytes": ([_I] * 5, _Z),
    "ttt_memo_mix_fwd": ([_I] * 7 + [_P] * 4 + [_I] + [_P] * 4 + [_P, _P, _I] + [_P, _P, _Z, _P], _I),
    "ttt_memo_mix_bwd": ([_I] * 7 + [_P] * 4 + [_I] + [_P] * 4 + [_P, _P, _I] + [_P] * 4 + [_P, _Z, _I, _P], _I),
    "ttt_prologue_fwd": ([_I] * 5 + [_P, _I, _L] + [_P] * 4 + [ctypes.c_float] + [_P] * 6, _I),
    "ttt_prologue_bwd": ([_I] * 5 + [_P, _I, _L] + [_P] * 4 + [ctypes.c_float] + [_P] * 10, _I),
    "ttt_post_norm_fwd": ([_I] * 4 + [_P, _I, _P, _P, ctypes.c_float, _P, _P], _I),
    "ttt_post_norm_bwd": ([_I] * 4 + [_P, _I, _P, _P, ctypes.c_float] + [_P] * 7, _I),
    "ttt_mlp_cached_readout": (
        [_I] * 6 + [_P, _I] + [_P, _L, _L] * 4 + [_P, _P, _I, _P, _P],
        _I,
    ),
}


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build the CUDA library first (python ttt-triton_b200/build.py); "
            "this package has no CPU or Triton fallback"
        )
    lib = ctypes.CDLL(LIB_PATH)
    for name, (args, res) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    return lib


lib = _load()


def exported_symbols():
    """Names of the C-ABI entry points this binding expects (all must resolve)."""
    return list(_SIGNATURES)


def launch_count():
    """Kernels this process has enqueued through the library (ttt_kernel_launches)."""
    return int(lib.ttt_kernel_launches())


def check(rc, name):
    if rc != 0:
        msg = lib.ttt_last_error().decode(errors="replace")
        raise RuntimeError(f"{name} failed (status {rc}): {msg}")


def device_status():
    """Read and clear the device error word (synchronises with the current device)."""
    v = ctypes.c_uint(0)
    check(lib.ttt_device_status(ctypes.byref(v)), "ttt_device_status")
    return v.value


def hold_first_stage(enable, wait_limit_ns=0):
    """Test switch of the bounded waits (ttt_test_hold_first_stage in include/ttt_b200.h)."""
    check(lib.ttt_test_hold_first_stage(int(bool(enable)), int(wait_limit_ns)), "ttt_test_hold_first_stage")


def set_forward_schedule(balanced, paired_ratio_milli=0):
    """Schedule switch of the tensor-core MLP forward (ttt_set_forward_schedule in
    include/ttt_b200.h): balanced two-launch schedule on (default) or off."""
    check(lib.ttt_set_forward_schedule(int(bool(balanced)), int(paired_ratio_milli)), "ttt_set_forward_schedule")


def forward_schedule_plan(streams, NC, num_sms, paired_ratio_milli=0):
    """(launches, rows) of the tensor-core MLP forward's balanced schedule for these sizes
    (ttt_mlp_fwd_schedule_plan; host only): rows are (launch, CTA, engine, stream, n0, n1)."""
    launches, n = ctypes.c_int(0), ctypes.c_int(0)
    cap = 4 * int(num_sms) + 8
    buf = (ctypes.c_int * (6 * cap))()
    check(lib.ttt_mlp_fwd_schedule_plan(int(streams), int(NC), int(num_sms), int(paired_ratio_milli),
                                        ctypes.byref(launches), buf, cap, ctypes.byref(n)),
          "ttt_mlp_fwd_schedule_plan")
    return launches.value, [tuple(buf[6 * k:6 * k + 6]) for k in range(n.value)]


def dtype_code(t):
    try:
        return DTYPE_CODES[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}; expected float32, bfloat16 or float16") from None


def ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def stream_of(t):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def require_cuda(*tensors):
    dev = None
    for t in tensors:
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"expected a torch.Tensor, got {type(t).__name__}")
        if not t.is_cuda:
            raise RuntimeError(
                "ttt-b200 kernels need CUDA tensors (there is no CPU fallback); got a tensor on " + str(t.device)
            )
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"all tensors must be on one device, got {dev} and {t.device}")
    return dev
