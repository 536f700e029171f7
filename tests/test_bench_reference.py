"""`bench.py --impl reference` on CPU: the reference arm times the
reference's own host kernels (its native C++ built from source into
oracle/_ref, else the oracle port) and prints one JSON line with the same
metric, unit and config as the GPU arm."""

from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--workload", "q8_0",
                        "--steps", "2", "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=REPO)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["metric"].startswith("weight-stream HBM GB/s") and d["value"] > 0
    assert d["steps"] == 2 and d["warmup"] == 3 and d["n_gpus"] == 1
    assert d["config"]["workload"].startswith("config 1: Q8_0 4096x4096")
    sys.path.insert(0, REPO)
    import bench
    wl = bench.WORKLOADS["q8_0"]
    # the GPU arm prints the same config dict (the driver compares them)
    assert d["config"] == bench.config_of(wl, wl["mats"], wl["batch"], 1, "weak")
    assert d["cpu_baseline"]["kind"] in ("reference", "port") and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_strong_scaling_shards_whole_layer():
    """The config-5 workload splits each projection's rows over the ranks;
    the shards of all ranks add back to the whole layer's bytes."""
    sys.path.insert(0, REPO)
    import bench

    mats = bench.WORKLOADS["layer_llama70b"]["mats"]
    assert bench.WORKLOADS["layer_llama70b"]["strong"]
    full = bench.algorithmic_bytes(mats, 1)
    for world in (1, 2, 4, 8):
        local = bench.shard_rows(mats, world)
        assert [m[2] * world for m in local] == [m[2] for m in mats]
        weights = sum(bench.synth.weight_bytes(q, n, k) for _, q, n, k, _ in local) * world
        assert weights == sum(bench.synth.weight_bytes(q, n, k) for _, q, n, k, _ in mats)
    assert full > 480e6
    with pytest.raises(ValueError):
        bench.shard_rows(mats, 3)


def test_cpu_leg_samples_rows_within_budget():
    """The CPU legs time whole-row samples sized to a time budget and scale
    the median back to the full workload by bytes."""
    sys.path.insert(0, REPO)
    import bench

    mats = [("w", "Q8_0", 512, 1024, "w"), ("v", "Q4_K", 256, 1024, "v")]
    host_w = bench.make_host_layer(mats, 0)
    sm, sw = bench.sample_rows(mats, host_w, 0.1)
    assert [m[2] for m in sm] == [52, 26]
    assert [w.nbytes for w in sw] == [52 * 34 * 32, 26 * 144 * 4]
    xs = [bench.synth.make_x(k, seed=1) for _, _, _, k, _ in mats]
    import time
    t0 = time.perf_counter()
    t_full, kind, desc = bench.cpu_leg(mats, 1, host_w, xs, "numpy", steps=3, warmup=1, budget_s=0.5)
    assert time.perf_counter() - t0 < 10 and t_full > 0 and kind == "port"
    assert "% of every projection's rows" in desc
