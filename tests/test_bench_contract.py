"""CPU: the tables and pure helpers of bench.py that the benchmark line is built from."""

import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

import bench  # noqa: E402


def test_records_and_traffic_name_real_workloads():
    for workload, key, metric in bench.FWDBWD_RECORDS:
        w = bench.WORKLOADS[workload]
        assert w["bwd"] and key.startswith("fwdbwd") and "fwd+bwd" in metric
    for (workload, kernel), (nbytes, tokens, source) in bench.NCU_TRAFFIC.items():
        w = bench.WORKLOADS[workload]
        assert kernel == w["kind"] + ("_bwd" if w["bwd"] else "_fwd")
        # captured at the workload's shape or a smaller batch of it (traffic scales with tokens)
        assert tokens % (w["NH"] * w["L"]) == 0 and tokens <= w["B"] * w["NH"] * w["L"] and nbytes > 0
        assert os.path.exists(os.path.join(os.path.dirname(HERE), source)), source


def test_algorithmic_figures_match_the_documented_ones():
    """544 / 960 B per token (bf16), 249,856 / 684,032 FLOP per token for the MLP and
    28,672 / 77,824 for the Linear scan (F 64, FF 256, CS 16)."""
    mlp = bench.algorithmic(bench.WORKLOADS["mlp_fwdbwd_c3"])
    assert mlp["fwd"] == (544, 249856) and mlp["bwd"] == (960, 684032)
    lin = bench.algorithmic(bench.WORKLOADS["linear_fwdbwd_c2"])
    assert lin["fwd"] == (544, 28672) and lin["bwd"] == (960, 77824)
    assert bench.algorithmic(bench.WORKLOADS["linear_fwd_c0"])["fwd"][0] == 1088  # fp32


def test_memo_segment_and_config_of_the_headline():
    w = bench.WORKLOADS["mlp_fwd_c1"]
    assert bench.memo_of(w) == w["L"] // bench.CS  # one memo state per stream
    assert bench.memo_of(bench.WORKLOADS["mlp_fwdbwd_c3"]) == 16

    class Args:
        workload = "mlp_fwd_c1"

    c = bench.ours_config(Args, w, 4)
    assert c["global_batch"] == 4 * w["B"] and c["B_per_rank"] == w["B"] and c["memo_segment_size"] == 128
    s = bench.ours_config(Args, dict(w, B=4), 4, sharded=True)
    assert "strong" in s["parallelism"]


def test_smi_index_follows_cuda_visible_devices(monkeypatch):
    import torch

    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "3,5")
    assert bench.smi_index(torch.device("cuda", 1)) == 5
    monkeypatch.delenv("CUDA_VISIBLE_DEVICES")
    assert bench.smi_index(torch.device("cuda", 1)) == 1
