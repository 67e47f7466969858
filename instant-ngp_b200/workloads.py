"""Seeded synthetic workloads standing in for the BASELINE configurations (numpy, host side).

The reference measures on NeRF-synthetic scenes that are not available here; these generators
produce inputs with the configurations' shapes, sizes and value distributions instead.  Every
generator takes a seed and returns host numpy arrays, so the CUDA library, the reference build
and the CPU oracle all see identical bytes.
"""
from __future__ import annotations

import math

import numpy as np


def encode_inputs(n: int, n_params: int, L: int, F: int, seed: int = 0, coord_stride: int = 3):
    """Config 0: n points uniform in [0,1)^3 (fp32 [n][coord_stride]), a U(-1e-4, 1e-4) fp16 table
    and dL/dy ~ N(0,1) rounded to fp16 in the feature-major [L*F][n] layout."""
    rng = np.random.default_rng(seed)
    coords = np.zeros((n, coord_stride), np.float32)
    coords[:, :3] = rng.random((n, 3), dtype=np.float32)
    if coord_stride >= 7:
        coords[:, 3] = math.sqrt(3.0) / 1024.0
        coords[:, 4:7] = 0.5
    table = (rng.random(n_params, dtype=np.float32) * 2e-4 - 1e-4).astype(np.float16)
    dy = rng.standard_normal((L * F, n), dtype=np.float32).astype(np.float16)
    return coords, table, dy
