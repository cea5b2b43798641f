"""CPU: the C-ABI library loads, exports every declared entry point, and rejects bad
arguments on the host (before any CUDA call), plus host-side checks of the Python layer."""

import ctypes
import os
import re

import pytest
import torch

import _lib

HDR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "ttt_b200.h")


def header_functions():
    text = open(HDR).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?(?:unsigned\s+)?(?:long\s+)*\w+\*?\s+\*?(ttt_\w+)\s*\(", text,
                                 flags=re.M)))


def test_header_declares_the_abi():
    names = header_functions()
    for want in ("ttt_linear_fwd", "ttt_linear_bwd", "ttt_mlp_fwd", "ttt_mlp_bwd", "ttt_mlp_cached_readout"):
        assert want in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    for name in header_functions():
        assert hasattr(lib, name), name
    assert sorted(_lib.exported_symbols()) == header_functions()
    assert _lib.lib.ttt_abi_version() == 10000


FAKE = ctypes.c_void_p(0x1000)  # never dereferenced: every call below fails its host checks first


def _linear_fwd(B=1, NH=1, NC=2, CS=16, F=16, ckpt=1, dt=0, null_out=False):
    return _lib.lib.ttt_linear_fwd(
        B, NH, NC, CS, F, ckpt, FAKE, FAKE, 0, FAKE, FAKE, FAKE, dt, FAKE, 0, FAKE, 0, FAKE, 0,
        None if null_out else FAKE, 0, FAKE, FAKE, FAKE, FAKE, None, None)


def test_host_checks_reject_bad_arguments():
    assert _linear_fwd(B=0) == -2
    assert "positive" in _lib.lib.ttt_last_error().decode()
    assert _linear_fwd(CS=15) == -2
    assert _linear_fwd(F=3) == -2
    assert _linear_fwd(ckpt=0) == -2
    assert _linear_fwd(dt=7) == -3
    assert _linear_fwd(null_out=True) == -1
    rc = _lib.lib.ttt_linear_bwd(1, 1, 4, 16, 16, 2, FAKE, FAKE, 0, FAKE, FAKE, FAKE, 0, FAKE, 0, FAKE, 0, FAKE, 0,
                                 FAKE, 0, None, None, None, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 0, FAKE,
                                 16, None)
    assert rc == -5 and "scratch" in _lib.lib.ttt_last_error().decode()


def test_scratch_sizes():
    assert _lib.lib.ttt_linear_bwd_scratch_bytes(2, 3, 10, 16, 64, 4) == 4 * 2 * 3 * 4 * 16 * 64
    assert _lib.lib.ttt_linear_bwd_scratch_bytes(2, 3, 3, 16, 64, 16) == 4 * 2 * 3 * 3 * 16 * 64  # group clamps to NC
    assert _lib.lib.ttt_mlp_bwd_scratch_bytes(1, 1, 8, 16, 64, 256, 4) == 4 * (2 * 64 * 256 + 4 * 16 * 320)
    assert _lib.lib.ttt_linear_bwd_scratch_bytes(0, 1, 1, 1, 1, 1) == 0


def test_python_layer_refuses_cpu_tensors():
    import ops

    x = torch.zeros(1, 1, 2, 16, 16)
    eta = torch.zeros(1, 1, 2, 16, 16)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        ops.ttt_linear(x, x, x, eta, torch.ones(1, 16), torch.zeros(1, 16), torch.zeros(1, 1, 16, 16),
                       torch.zeros(1, 1, 1, 16), 1)


def test_dtype_codes():
    assert _lib.dtype_code(torch.zeros(1)) == 0
    assert _lib.dtype_code(torch.zeros(1, dtype=torch.bfloat16)) == 1
    assert _lib.dtype_code(torch.zeros(1, dtype=torch.float16)) == 2
    with pytest.raises(TypeError):
        _lib.dtype_code(torch.zeros(1, dtype=torch.float64))


def test_noalloc_backward_rejects_requests_beyond_its_scratch():
    # 4096 streams x 16 x 16 x 64 fp32 = 64 MiB of scratch > the library's 16 MiB
    rc = _lib.lib.ttt_linear_bwd_noalloc(64, 64, 16, 16, 64, 16, FAKE, FAKE, 0, FAKE, FAKE, FAKE, 0, FAKE, 0, FAKE,
                                         0, FAKE, 0, FAKE, 0, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 0, None)
    assert rc == -5 and "16777216" in _lib.lib.ttt_last_error().decode()


def test_mlp_saved_preactivations_all_or_none():
    P = [FAKE] * 4
    rc = _lib.lib.ttt_mlp_fwd(1, 1, 2, 16, 64, 256, 1, 1, FAKE, FAKE, 0, *P, FAKE, 1, FAKE, 1, FAKE, 1, FAKE, 1,
                              FAKE, 1, *P, *P, None, None, None, None, FAKE, None, None, None, None)
    assert rc == -1 and "pre-activation" in _lib.lib.ttt_last_error().decode()

    def bwd(saved, scratch):
        return _lib.lib.ttt_mlp_bwd(1, 1, 2, 16, 64, 256, 1, FAKE, FAKE, 0, *P, FAKE, 1, FAKE, 1, FAKE, 1, FAKE, 1,
                                    FAKE, 1, *saved, *([FAKE] * 10), 1, scratch, 0, None)

    assert bwd([FAKE, None, None, None, None, None], None) == -1
    assert "all set or all NULL" in _lib.lib.ttt_last_error().decode()
    # without the saved pre-activations the recompute path needs its scratch buffer
    assert bwd([None] * 6, None) == -5


def test_device_status_rejects_null():
    assert _lib.lib.ttt_device_status(None) == -1


def test_memo_mix_host_checks():
    P = [FAKE] * 4

    def fwd(NC, M, F=64, dt=1, scratch=FAKE, nbytes=1 << 40):
        return _lib.lib.ttt_memo_mix_fwd(1, 1, NC, 16, F, 256, M, *P, dt, *P, FAKE, FAKE, 1, FAKE, scratch, nbytes,
                                         None)

    assert fwd(8, 0) == -2
    assert fwd(8, 2, F=32) == -4 and "F = 64" in _lib.lib.ttt_last_error().decode()
    assert fwd(130, 2) == -4 and "at most 64" in _lib.lib.ttt_last_error().decode()
    assert fwd(8, 2, dt=0) == -3
    assert fwd(8, 2, scratch=None) == -1
    assert fwd(8, 2, nbytes=16) == -5
    # fp32 memo states are read with 16-byte accesses: each of the four must be 16-byte aligned
    odd = ctypes.c_void_p(0x1004)
    for i in range(4):
        memo = [FAKE] * 4
        memo[i] = odd
        rc = _lib.lib.ttt_memo_mix_fwd(1, 1, 8, 16, 64, 64, 2, *P, 1, *memo, FAKE, FAKE, 1, FAKE, FAKE, 1 << 40, None)
        assert rc == -7 and "memo states" in _lib.lib.ttt_last_error().decode()
    # W1/W2 16-bit copies (2 * F * FF * 2 bytes) plus summary and its gradient (2 * F * 4) per memo state
    assert _lib.lib.ttt_memo_mix_scratch_bytes(2, 3, 9, 4, 256) == 2 * 3 * 3 * (2 * 64 * 256 * 2 + 2 * 64 * 4)
    assert _lib.lib.ttt_memo_mix_scratch_bytes(2, 3, 9, 4, 64) == 2 * 3 * 3 * (2 * 64 * 64 * 2 + 2 * 64 * 4)


def test_prologue_host_checks():
    """ttt_prologue_fwd / _bwd reject bad sizes, strides, dtypes and alignment on the host."""
    A = ctypes.c_void_p(0x1000)

    def fwd(B=2, L=32, NH=4, F=64, CS=16, P=A, dt=1, ld=4 * 4 * 64 + 8, out=A):
        return _lib.lib.ttt_prologue_fwd(B, L, NH, F, CS, P, dt, ld, A, A, A, A, 0.1, out, out, out, out, out, None)

    assert fwd(P=None) == -1
    assert fwd(out=None) == -1
    assert fwd(F=48) == -2 and "head_dim" in _lib.lib.ttt_last_error().decode()
    assert fwd(L=40) == -2 and "multiple" in _lib.lib.ttt_last_error().decode()
    assert fwd(dt=9) == -3
    assert fwd(ld=4 * 4 * 64) == -2  # no room for the gate columns
    assert fwd(ld=4 * 4 * 64 + 6) == -2  # not a multiple of 8
    assert fwd(P=ctypes.c_void_p(0x1002)) == -7
    rc = _lib.lib.ttt_prologue_bwd(1, 16, 4, 64, 16, A, 1, 4 * 4 * 64 + 8, A, A, A, A, 0.1, None, None, None, None,
                                   None, None, A, A, None, None)
    assert rc == -1  # dproj is required; the incoming gradients may all be NULL


def test_post_norm_host_checks():
    A = ctypes.c_void_p(0x1000)

    def fwd(B=2, NH=4, L=32, F=64, X=A, dt=1, eps=1e-6, Y=A):
        return _lib.lib.ttt_post_norm_fwd(B, NH, L, F, X, dt, A, A, eps, Y, None)

    assert fwd(X=None) == -1
    assert fwd(Y=None) == -1
    assert fwd(F=60) == -2 and "multiple" in _lib.lib.ttt_last_error().decode()
    assert fwd(NH=32) == -2 and "width" in _lib.lib.ttt_last_error().decode()
    assert fwd(dt=0, NH=16) == -2  # 1024 fp32 columns exceed the fp32 limit
    assert fwd(dt=4) == -3
    assert fwd(eps=-1.0) == -2
    assert fwd(X=ctypes.c_void_p(0x1008)) == -7
    assert _lib.lib.ttt_post_norm_bwd(2, 4, 32, 64, A, 1, A, A, 1e-6, None, A, A, A, None, None, None) == -1
    assert _lib.lib.ttt_post_norm_bwd(2, 4, 32, 64, A, 1, A, A, 1e-6, A, A, A, A, A, None, None) == -1


def test_noalloc_backward_rejects_requests_beyond_its_fixed_scratch():
    """ttt_linear_bwd_noalloc checks the scratch its sizes need against the library's fixed
    16 MiB array before any CUDA call: a request twice the array (batch 64, 8 heads, group 16) is refused with
    TTT_ERR_SCRATCH and a message naming both sizes."""
    def call(B, NH, NC, ckpt):
        return _lib.lib.ttt_linear_bwd_noalloc(
            B, NH, NC, 16, 64, ckpt, FAKE, FAKE, 0, FAKE, FAKE, FAKE, 1, FAKE, 1, FAKE, 1, FAKE, 1, FAKE, 1,
            FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 1, None)

    need = _lib.lib.ttt_linear_bwd_scratch_bytes(64, 8, 256, 16, 64, 16)
    assert need > 16 << 20
    assert call(64, 8, 256, 16) == -5
    msg = _lib.lib.ttt_last_error().decode()
    assert str(need) in msg and str(16 << 20) in msg
    assert call(0, 8, 256, 16) == -2  # the shape checks run first
