"""Host-side helpers of bench.py that shape the reported numbers (no GPU): the roofline entry of
the dominant kernel with its DRAM traffic scaled from an ncu capture, and the OpenMP thread
share that torchrun ranks get for the engine's set-up."""
import json
import os
import sys

import pytest

from conftest import ROOT

sys.path.insert(0, ROOT)
import bench  # noqa: E402


def test_roofline_picks_the_dominant_kernel_and_scales_traffic():
    # {name: (launches, total ms, algorithmic bytes)}; op:* entries are inclusive scopes, never the kernel
    N = 1 << 16
    prof = {"op:bootstrap": (10, 9000.0, 0.0),
            "ntt_fwd": (100, 50.0, 100 * 40 * 16.0 * N),      # 40 limbs per launch on average
            "key_inner": (100, 20.0, 1e9)}
    r = bench.roofline(prof)
    assert r["kernel"] == "ntt_fwd" and r["bound"] == "hbm" and r["unit"] == "GB/s"
    assert r["achieved"] == pytest.approx(100 * 40 * 16.0 * N / 0.050 / 1e9)
    assert r["frac"] == pytest.approx(r["achieved"] / r["peak"])
    assert r["avg_launch_us"] == pytest.approx(500.0)
    t = json.load(open(os.path.join(ROOT, "profiles", "traffic.json")))["ntt_fwd"]
    # captured DRAM bytes per limb times the run's own limbs per launch
    assert r["traffic"] == pytest.approx(t["dram_bytes_per_limb"] * 40)
    assert t["dram_bytes_per_limb"] > t["algorithmic_bytes_per_limb"]   # the two-phase transform re-reads


def test_aggregate_throughput_counts_every_rank():
    assert bench.aggregate_tokens_per_s(64, 4, 2, 8000.0) == pytest.approx(64 * 4 * 2 / 8.0)


def test_torchrun_ranks_share_the_host_cores(monkeypatch):
    monkeypatch.setenv("LOCAL_WORLD_SIZE", "4")
    monkeypatch.setenv("OMP_NUM_THREADS", "1")
    bench.host_threads()
    assert int(os.environ["OMP_NUM_THREADS"]) == max(1, (os.cpu_count() or 1) // 4)
    monkeypatch.setenv("LOCAL_WORLD_SIZE", "1")
    monkeypatch.setenv("OMP_NUM_THREADS", "1")
    bench.host_threads()
    assert os.environ["OMP_NUM_THREADS"] == "1"    # a single process keeps what it was given
