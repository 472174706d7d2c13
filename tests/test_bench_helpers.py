"""The benchmark's bookkeeping, on the CPU: roofline arithmetic, configs, traffic.

``bench.py`` prints one JSON line whose numbers a reader checks by hand:
achieved = algorithmic bytes per launch / average launch duration, frac =
achieved / the measured copy peak, the ``config`` that both arms print, and
the DRAM traffic scaled from the committed ncu summary.  These tests pin that
arithmetic without a GPU.
"""

from __future__ import annotations

import json
from pathlib import Path

import pytest

import bench
from marathon_b200.workloads import config

ROOT = Path(__file__).resolve().parents[1]


def test_roofline_is_bytes_over_launch_time_against_the_measured_peak():
    peak, kind = bench.peaks()
    measured = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["hbm_gbs"]
    assert (peak, kind) == (float(measured), "measured")
    cfg = config("c2")
    r = bench.roofline(cfg.algorithmic_bytes(), 1.4, None, "move_kernel<load>")
    assert r["bytes_per_launch"] == 28_608 * 40 * 8_192
    assert r["achieved"] == pytest.approx(9.37426944e9 / 1.4e-3 / 1e9, abs=0.1)
    assert r["frac"] == pytest.approx(r["achieved"] / peak, abs=1e-4)
    assert r["frac_of_8tbs"] == pytest.approx(r["achieved"] / 8000.0, abs=1e-4)
    assert r["bound"] == "hbm" and r["unit"] == "GB/s" and r["traffic"] is None


def test_both_arms_print_the_same_config():
    cfg = config("c2")
    for world in (1, 2, 4, 8):
        a = bench.workload_config(cfg, world, "nhd")
        assert a == bench.workload_config(cfg, world, "nhd")
        assert a["turn_bytes"] == cfg.algorithmic_bytes()
        assert a["heads_per_rank"] == 8 // world
        assert a["parallelism"] == f"kv-head shard tp{world}"
        assert "model" not in a  # a workload, not a model


def test_rank_share_reports_only_that_share():
    cfg = config("c2")
    share = bench.workload_config(cfg, 1, "nhd", 8)
    assert share["heads_per_rank"] == 1
    assert share["turn_bytes"] == cfg.algorithmic_bytes() // 8 == 1_171_783_680
    assert "share of 8" in share["workload"] and "one GPU" in share["parallelism"]


@pytest.mark.parametrize("name", ["c2", "c3"])
def test_traffic_scales_the_committed_ncu_figure_by_units(name):
    rec = json.loads((ROOT / "profiles" / "traffic.json").read_text())[f"{name}/nhd"]
    cfg = config(name)
    units = cfg.shifted_tokens * cfg.layers
    assert rec["units"] == units
    full = bench.traffic_for(name, "nhd", units)
    assert full == pytest.approx(rec["dram_bytes"])
    assert bench.traffic_for(name, "nhd", units // 2) == pytest.approx(rec["dram_bytes"] / 2)
    # reads are the algorithmic reads; some writes are still in L2 at kernel end
    algorithmic = cfg.algorithmic_bytes()
    assert rec["dram_read_bytes"] == pytest.approx(algorithmic / 2, rel=1e-3)
    assert 0.97 * algorithmic < full <= algorithmic * 1.001
    assert bench.traffic_for(name, "hnd", units) is None  # no summary for that layout


def test_bench_ring_is_deeper_than_the_library_default():
    from marathon_b200.shift_kernels import Launcher

    default = Launcher.__init__.__defaults__[-1]
    assert bench.BENCH_SLOTS > default == 4
