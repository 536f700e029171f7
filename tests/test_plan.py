"""Launch plans of the tensor-core batch-1 kernel, checked on the host (no
GPU): frc_batch1_plan returns the configuration a launch would use, and the
properties every launch relies on for staying inside its buffers and for
finishing hold over a grid of shapes and device sizes.

* the dynamic shared memory fits the 227 KB a CTA may opt into;
* a split launch (rows in parts of k on thread-block clusters) has one part
  per CTA, no builder warps, at most 8 CTAs per cluster (the portable
  size), and CTAs = CTAs per cluster x row ranges <= SMs; its row ranges
  hold every row even when only half of them are resident at once (the
  launch runs no more ranges than the device holds clusters);
* a one-CTA-per-range launch has at most one CTA per SM and its CTAs hold
  every row;
* no part of k is empty."""

from __future__ import annotations

import pytest

from flatrun_b200 import _lib

SMEM_OPT_IN = 227 * 1024
KS = [256, 512, 2304, 3584, 4096, 5120, 8192, 14336, 18944, 28672, 36864, 49152, 65536, 131072]
NS = [1, 7, 16, 17, 33, 300, 1024, 1280, 2048, 2368, 2400, 3584, 4096, 8192, 57344, 152064]


def _ceil(a, b):
    return (a + b - 1) // b


@pytest.mark.parametrize("quant", ["Q4_K", "Q5_K"])
@pytest.mark.parametrize("sms", [148, 132, 8, 2, 1])
def test_tensor_core_plans_stay_inside_their_buffers(quant, sms):
    tensor = 0
    for k in KS:
        for n in NS:
            p = _lib.batch1_plan(quant, n, k, sms)
            if p["kernel"] != "tensor_fp32":
                continue
            tensor += 1
            where = (quant, n, k, sms, p)
            assert 0 < p["smem"] <= SMEM_OPT_IN, where
            assert p["stages"] >= 2, where
            assert p["tiles_per_warp"] in (1, 2), where
            parts = _ceil(p["chunks"], p["part_chunks"])
            assert (parts - 1) * p["part_chunks"] < p["chunks"], where  # no empty part
            if p["split"] > 1:
                assert 2 <= p["split"] <= 8 and p["split"] == parts, where
                assert p["builders"] == 0 and p["tiles_per_warp"] == 2 and p["warps"] <= 8, where
                assert p["ctas"] == p["split"] * p["ranges"] <= sms, where
                assert _ceil(n, max(1, p["ranges"] // 2)) <= p["rows_max"], where
            else:
                assert 1 <= p["ctas"] <= sms, where
                assert _ceil(n, p["ctas"]) <= p["rows_max"], where
    assert tensor > 0


def test_plans_of_the_benchmarked_shapes():
    """The shapes the design notes quote: Llama-3-70B gate+up on 148 SMs
    (11 warps, three chunks, one part), its down projection (two parts of 7
    chunks on clusters of two, 74 ranges), the same down shard at 1024 rows
    (16-row CTAs: 64 ranges), and a 1024-row k = 8192 shard on 64 CTAs."""
    g = _lib.batch1_plan("Q4_K", 57344, 8192)
    assert (g["kernel"], g["warps"], g["chunks"], g["split"], g["ctas"]) == ("tensor_fp32", 11, 3, 1, 148)
    d = _lib.batch1_plan("Q4_K", 8192, 28672)
    assert (d["warps"], d["chunks"], d["part_chunks"], d["split"], d["ranges"], d["ctas"]) == (8, 14, 7, 2, 74, 148)
    assert _lib.batch1_plan("Q4_K", 1024, 28672)["ranges"] == 64
    assert _lib.batch1_plan("Q4_K", 1024, 8192)["ctas"] == 64
    assert _lib.batch1_plan("Q6_K", 4096, 4096)["kernel"] == "cuda_core_fp32"


def test_plan_argument_errors():
    lib = _lib.load()
    import ctypes
    arr = (ctypes.c_int64 * len(_lib.PLAN_FIELDS))()
    assert lib.frc_batch1_plan(_lib.QUANT_IDS["Q4_K"], 0, 4096, 148, arr) == _lib.FRC_ERR_INVALID
    assert lib.frc_batch1_plan(_lib.QUANT_IDS["Q4_K"], 16, 4097, 148, arr) == _lib.FRC_ERR_INVALID
    assert lib.frc_batch1_plan(_lib.QUANT_IDS["Q4_K"], 16, 4096, 0, arr) == _lib.FRC_ERR_INVALID
