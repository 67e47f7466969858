"""Host-side rules of the trainer against the reference's formulas (no GPU needed)."""
from __future__ import annotations

import numpy as np


def _reference_adaptive_batch(rays, before, measured):
    """ngp.train.cpp:132-133 written out: granule 128, batch 2^18, MAX_SAMPLES 2^22."""
    g, batch, max_samples = 128, 1 << 18, 1 << 22
    infer = ((min(before, max_samples) + g - 1) // g) * g
    want = min((rays * batch) // measured, batch)
    return min(max(((want + g - 1) // g) * g, g), batch), infer


def test_adaptive_batch_rule_matches_reference(ngp):
    rng = np.random.default_rng(0)
    cases = [(4096, 1_400_000, 262_144), (128, 10, 1), (1 << 18, 1 << 24, 1 << 18), (12160, 1_433_429, 263_000), (128, 0, 1 << 30)]
    cases += [(int(rng.integers(128, 1 << 18)), int(rng.integers(0, 1 << 25)), int(rng.integers(1, 1 << 20))) for _ in range(2000)]
    for rays, before, measured in cases:
        assert ngp.adaptive_batch(rays, before, measured) == _reference_adaptive_batch(rays, before, measured), (rays, before, measured)
