"""Per-phase timeline of the TTT-MLP tensor-core forward (one mini-batch, every CTA) and the
steady-state time per mini-batch of every stream.

    python ttt-triton_b200/build.py --phase-stamps
    python ttt-triton_b200/phase_timeline.py [--batch B] [--plain]
    python ttt-triton_b200/phase_timeline.py --backward --batch 9

With --backward it times the MLP backward's reverse walk instead (config 3's heads and
length, FF 256, bf16): the median time of each phase of walk step 64, phases R1 / M1 / R2 /
M2 / R3 as in ttt_mlp_bwd_tc.cu.

Runs the config-1 forward (B x 12 heads, L 2048, F 64, FF 256, bf16, memo states every 16
mini-batches) on libttt_b200_stamps.so. That build records, on thread 0 of every stream's
warps, %globaltimer at the loop top of mini-batches n0 + 4 and n1 - 4 of its range, which
gives each stream's steady-state time per mini-batch (printed per launch, for streams alone
on their SM and streams sharing it). With --plain (one CTA per stream: the balanced
two-launch schedule switched off) it also records before and after each CTA barrier of
mini-batch 64 and prints the median time of each phase, separately for CTAs alone on their
SM and CTAs sharing it. Phases: A = the first MMA phase (Z1, XQ W1, GELU, partial Z2),
C = the LayerNorm-gradient row phase, D = the second MMA phase (G1, the updates, the
dual-form read-out products), E = the read-out LayerNorm row phase; "sync" = the wait at the
barrier that ends a phase.
"""

from __future__ import annotations

import argparse
import collections
import ctypes
import os
import statistics
import sys

os.environ["TTT_B200_LIB"] = "libttt_b200_stamps.so"
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

import torch  # noqa: E402

import _core  # noqa: E402
import _lib  # noqa: E402
import synthetic as S  # noqa: E402

PHASES = ("top barrier", "A", "A sync", "C", "C sync", "D", "D sync", "E")
NAMES = ("ln_w", "ln_b", "W1", "b1", "W2", "b2", "XQ", "XV", "XK", "eta")


def rates(n_rows, balanced, M, S_):
    """Median steady-state ns per mini-batch of each launch, streams alone / sharing an SM."""
    read = _lib.lib.ttt_rate_stamps_read
    read.argtypes, read.restype = [ctypes.c_void_p, ctypes.c_int], ctypes.c_int
    buf = (ctypes.c_ulonglong * (2 * n_rows * 4))()
    if read(buf, n_rows) != 0:
        raise RuntimeError("reading the rate stamps failed (is this the --phase-stamps build?)")
    R = [[[buf[(l * n_rows + i) * 4 + k] for k in range(4)] for i in range(n_rows)] for l in range(2)]
    if not balanced:
        per_sm = collections.Counter(r[3] for r in R[0])
        groups = [("launch", "alone", [r for r in R[0] if per_sm[r[3]] == 1]),
                  ("launch", "sharing", [r for r in R[0] if per_sm[r[3]] > 1])]
    else:
        D = S_ - M  # CTAs 0..D-1 run two streams (rows 2c, 2c+1); the rest one (row 2c)
        groups = []
        for l in range(2):
            groups += [(f"launch {l + 1}", "sharing", [R[l][2 * c + e] for c in range(D) for e in range(2)]),
                       (f"launch {l + 1}", "alone", [R[l][2 * c] for c in range(D, M)])]
    for launch, label, sel in groups:
        sel = [r for r in sel if r[2] > 0]
        if sel:
            v = statistics.median((r[1] - r[0]) / r[2] for r in sel)
            print(f"  {launch}, {label} ({len(sel)} streams): {v:.0f} ns per mini-batch")


BWD_PHASES = ("loop top (stage wait + barrier)", "R1", "R1 barrier", "M1", "M1 barrier", "R2", "R2 barrier",
              "M2", "M2 barrier", "R3")


def backward(B, NH, NC):
    """Per-phase timeline of step 64 of the MLP backward's reverse walk (FF 256, bf16): median
    over CTAs of each phase (ns), from the stamps of thread 0 of every CTA."""
    d = S.make_mlp_inputs(B, NH, NC, 16, 64, 256, dtype=torch.bfloat16, device="cuda", seed=0)
    dO = S.make_upstream((B, NH, NC, 16, 64), device="cuda", seed=1, dtype=torch.bfloat16)
    _, last, ck, _, zs = _core.mlp_forward(*(d[k] for k in NAMES), 16, None)

    def step():
        _core.mlp_backward(d["ln_w"], d["ln_b"], ck, d["XQ"], d["XV"], d["XK"], d["eta"], dO, 16, saved=zs,
                           W1_last=last[0], W2_last=last[2])

    for _ in range(2):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    step()
    e1.record()
    torch.cuda.synchronize()
    read = _lib.lib.ttt_bwd_phase_stamps_read
    read.argtypes, read.restype = [ctypes.c_void_p, ctypes.c_int], ctypes.c_int
    n = B * NH
    buf = (ctypes.c_ulonglong * (12 * n))()
    if read(buf, n) != 0:
        raise RuntimeError("reading the timeline failed (is this the --phase-stamps build?)")
    rows = [[buf[i * 12 + k] for k in range(12)] for i in range(n)]
    rows = [r for r in rows if r[0] and r[10]]
    print(f"backward B={B} NH={NH} NC={NC}: {e0.elapsed_time(e1):.3f} ms per launch, {len(rows)} CTAs stamped")
    for k, name in enumerate(BWD_PHASES):
        v = [r[k + 1] - r[k] for r in rows if r[k] and r[k + 1]]
        if v:
            print(f"  {name:32s} {statistics.median(v):7.0f} ns")
    print(f"  {'step':32s} {statistics.median(r[10] - r[0] for r in rows):7.0f} ns")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--plain", action="store_true", help="one CTA per stream (balanced schedule off)")
    ap.add_argument("--backward", action="store_true",
                    help="the MLP backward instead: config-3 heads and length (NH 16, L 8192) at --batch")
    args = ap.parse_args()
    if args.backward:
        backward(args.batch, 16, 512)
        return
    read = _lib.lib.ttt_phase_stamps_read
    read.argtypes, read.restype = [ctypes.c_void_p, ctypes.c_int], ctypes.c_int
    B, NH = args.batch, 12
    M = torch.cuda.get_device_properties(0).multi_processor_count
    n = B * NH
    balanced = not args.plain and M < n <= M + M // 3
    _lib.set_forward_schedule(not args.plain)
    d = S.make_mlp_inputs(B, NH, 128, 16, 64, 256, dtype=torch.bfloat16, device="cuda", seed=0)
    for _ in range(3):
        _core.mlp_forward(*(d[k] for k in NAMES), 16, 16, for_backward=False)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(5):
        _core.mlp_forward(*(d[k] for k in NAMES), 16, 16, for_backward=False)
    e1.record()
    torch.cuda.synchronize()
    print(f"B={B}: {n} streams, {e0.elapsed_time(e1) / 5:.4f} ms per forward"
          + (" (balanced two-launch schedule)" if balanced else ""))
    rates(2 * M if balanced else n, balanced, M, n)
    if balanced:
        return
    buf = (ctypes.c_ulonglong * (10 * n))()
    if read(buf, n) != 0:
        raise RuntimeError("reading the timeline failed (is this the --phase-stamps build?)")
    rows = [[buf[i * 10 + k] for k in range(10)] for i in range(n)]
    per_sm = collections.Counter(r[9] for r in rows)
    for label, sel in (("alone on its SM", [r for r in rows if per_sm[r[9]] == 1]),
                       ("sharing its SM", [r for r in rows if per_sm[r[9]] > 1])):
        if not sel:
            continue
        total = statistics.median(r[8] - r[0] for r in sel)
        print(f"{label}: {len(sel)} CTAs, mini-batch {total:.0f} ns (median)")
        for k, name in enumerate(PHASES):
            print(f"  {name:12s} {statistics.median(r[k + 1] - r[k] for r in sel):7.0f} ns")


if __name__ == "__main__":
    main()
