"""Final-PSNR parity with the reference (north_star: within 0.2 dB).

The reference's own training loop (InstantNGP::train, ngp.train.cpp:108-155, replayed through its
ngp::cuda interface by oracle/train_replay.inc on the reference's compiled ngp.train.cu) and this
library's trainer (InstantNGP, at the reference's compiled layout: 8 levels x 4 features, log2 T
19, scale 2) train on the same config-3 scene -- 100 train and 20 test views of 800 x 800, the
seeded 64-sphere scene -- for 2000 steps each, on three scenes (seeds).  Test PSNR is computed the
reference's way (ngp.train.cpp:183-229: SSE over the test images against the sRGB targets).

Sample placement (ray order vs atomic order), fp32 vs fp16 gradient sums and fp32 vs fp16
network accumulation make single runs differ; the bar is on the mean over the scenes: the
library's mean test PSNR is at least the reference's minus 0.2 dB, and the mean absolute
difference is reported (printed) beside it.
"""
from __future__ import annotations

import numpy as np
import pytest

import workloads

pytestmark = pytest.mark.gpu

STEPS = 2000
SEEDS = (3, 13, 23)


def _reference_psnr(scene) -> float:
    from oracle import REF_SO, ReplayTrainer

    t = ReplayTrainer(REF_SO, scene["train"], scene["test"])
    try:
        t.train(STEPS)
        return float(t.test_psnr())
    finally:
        t.close()


def _library_psnr(ngp, scene) -> float:
    model = ngp.InstantNGP(scene, ngp.trainer_config())
    try:
        model.train(STEPS)
        return float(model.test()["psnr"])
    finally:
        model.close()


def test_final_psnr_matches_reference_over_three_scenes(ngp, reflib):
    ours, ref = [], []
    for seed in SEEDS:
        scene = workloads.procedural_dataset(n_train=100, n_test=20, width=800, height=800, seed=seed, device="cuda")
        ref.append(_reference_psnr(scene))
        ours.append(_library_psnr(ngp, scene))
    delta = np.array(ours) - np.array(ref)
    print(f"test PSNR after {STEPS} steps: library {np.round(ours, 3).tolist()} reference {np.round(ref, 3).tolist()} "
          f"delta {np.round(delta, 3).tolist()} mean {delta.mean():+.3f} dB")
    assert min(ours) > 20.0
    assert delta.mean() >= -0.2
