"""Build libttt_b200.so in-tree with nvcc for sm_100a.

    python ttt-triton_b200/build.py [--force] [--phase-stamps]

The library is a plain C-ABI shared object (include/ttt_b200.h); nothing here links
against torch. The build is incremental on source modification times. ``--phase-stamps``
builds a second library, libttt_b200_stamps.so, whose TTT-MLP tensor-core forward records a
per-phase %globaltimer timeline (phase_timeline.py reads it); the product library has none.
"""

from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libttt_b200.so")
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
]


def _nvcc():
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libttt_b200.so")
    return cand


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


STAMPS_LIB = os.path.join(HERE, "libttt_b200_stamps.so")


def _stale(lib=LIB):
    if not os.path.exists(lib):
        return True
    t = os.path.getmtime(lib)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(REPO, "include", "*.h"))
    return any(os.path.getmtime(d) > t for d in deps)


def build(force=False, verbose=False, phase_stamps=False):
    """Compile every .cu under csrc/ into libttt_b200.so (sm_100a), or with phase_stamps into
    libttt_b200_stamps.so with the forward's timeline stamps compiled in. Returns the path."""
    lib = STAMPS_LIB if phase_stamps else LIB
    if not force and not _stale(lib):
        return lib
    tmp = lib + ".tmp"
    extra = ["-DTTT_PHASE_STAMPS"] if phase_stamps else []
    cmd = [_nvcc(), *NVCC_FLAGS, *extra, "-I", os.path.join(REPO, "include"), "-o", tmp, *sources()]
    if verbose:
        print(" ".join(cmd))
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True, phase_stamps="--phase-stamps" in sys.argv))
