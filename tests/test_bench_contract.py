"""CPU tier: the host-side pieces of bench.py that shape its JSON line -- the training roofline's
choice of kernel and its arithmetic, and the peaks it divides by.  No GPU needed."""
from __future__ import annotations

import sys

import pytest

from conftest import ROOT

if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import bench  # noqa: E402

PEAKS = {"hbm_gbs": 6500.0, "bf16_tflops": 1600.0, "bf16_tflops_sustained": 1400.0, "source": "test"}
L2 = {"l2_read_GBps": 20000.0, "gather_GBps": 8000.0}


def phases(**ms):
    return {"steps": 10, "ms": {k: 10.0 * v for k, v in ms.items()}, "mean_inference_samples": 1_400_000}


def grid(updates=10, **ms):
    return {"updates": updates, "mean_samples": float(1 << 21), "ms": {k: updates * v for k, v in ms.items()}}


def test_roofline_names_the_longest_grid_kernel():
    r = bench.train_roofline(phases(grid_update=0.6, march=0.2, adam=0.07), grid(grid_samples=0.05, grid_encode=0.3, grid_density=0.1), PEAKS, L2)
    assert r["kernel"].startswith("encode_grid_samples_kernel") and r["bound"] == "hbm"
    # 68 algorithmic HBM bytes per grid sample (64 B features + 4 B cell index out) over the launch
    want = 68 * (1 << 21) / 0.3e-3 / 1e9
    assert r["achieved"] == pytest.approx(want, rel=1e-3)
    assert r["frac"] == pytest.approx(want / PEAKS["hbm_gbs"], rel=1e-2)
    assert 0 < r["share_of_step"] < 1
    l2 = r["l2"]
    assert l2["achieved"] == pytest.approx(512 * (1 << 21) / 0.3e-3 / 1e9, rel=1e-3)
    assert l2["frac_of_stream_read"] == pytest.approx(l2["achieved"] / L2["l2_read_GBps"], rel=1e-2)


def test_roofline_without_grid_updates_says_so():
    r = bench.train_roofline(phases(march=0.2), grid(updates=0), PEAKS, L2)
    assert r["kernel"] is None


def test_peaks_come_from_the_measured_file_or_the_stated_fallback():
    p = bench.load_peaks()
    assert p["source"] in ("measured", "fallback")
    assert p["hbm_gbs"] > 1000 and p["bf16_tflops"] > 100


def test_roofline_reports_the_request_path():
    r = bench.train_roofline(phases(grid_update=0.6, march=0.2, adam=0.07), grid(grid_samples=0.05, grid_encode=0.3, grid_density=0.1), PEAKS, L2)
    req = r["l2"]["requests"]
    per = bench.GRID_KERNELS["grid_encode"]["l2_requests"]
    assert req["achieved_G_per_s"] == pytest.approx(per * (1 << 21) / 0.3e-3 / 1e9, rel=1e-3)
    assert req["probe_G_per_s"] == pytest.approx(L2["gather_GBps"] / 4.0)
    assert req["frac"] == pytest.approx(req["achieved_G_per_s"] / req["probe_G_per_s"], rel=1e-2)
