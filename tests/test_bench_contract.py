"""CPU tier: the host-side pieces of bench.py that shape its JSON line -- the training roofline's
choice of phase and its arithmetic, and the peaks it divides by.  No GPU needed."""
from __future__ import annotations

import sys

import pytest

from conftest import ROOT

if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import bench  # noqa: E402

PEAKS = {"hbm_gbs": 6500.0, "bf16_tflops": 1600.0, "bf16_tflops_sustained": 1400.0, "source": "test"}


def phases(**ms):
    return {"steps": 10, "ms": {k: 10.0 * v for k, v in ms.items()}, "mean_inference_samples": 1_400_000}


def test_roofline_skips_the_overlapped_march():
    r = bench.phase_roofline(phases(march=0.30, inference_compact=0.25, encode_bwd=0.11, adam=0.07), PEAKS)
    assert r["phase"] == "inference_compact" and r["bound"] == "hbm"
    # 28 algorithmic bytes per marched sample over the phase's time
    want = 28 * 1_400_000 / 0.25e-3 / 1e9
    assert r["achieved"] == pytest.approx(want, rel=1e-3)
    assert r["frac"] == pytest.approx(want / PEAKS["hbm_gbs"], rel=1e-2)
    assert 0 < r["share"] < 1


def test_roofline_of_a_tensor_bound_phase():
    r = bench.phase_roofline(phases(march=0.1, mlp_bwd=0.5, adam=0.07), PEAKS)
    assert r["bound"] == "tensor" and r["unit"] == "TFLOP/s"
    want = bench.MLP_FWDBWD_FLOP * bench.BATCH / 0.5e-3 / 1e12
    assert r["achieved"] == pytest.approx(want, rel=1e-3)
    assert r["peak"] == PEAKS["bf16_tflops_sustained"]


def test_peaks_come_from_the_measured_file_or_the_stated_fallback():
    p = bench.load_peaks()
    assert p["source"] in ("measured", "fallback")
    assert p["hbm_gbs"] > 1000 and p["bf16_tflops"] > 100
