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


def xavier_mlp_params(seed: int = 0) -> np.ndarray:
    """Config 1: the 10,240 packed MLP weights, Xavier-uniform per matrix (fan_in + fan_out), fp16,
    in the reference's order and shapes (ngp.train.cu:1429-1452)."""
    rng = np.random.default_rng(seed)
    shapes = [(64, 32), (16, 64), (64, 32), (64, 64), (16, 64)]
    parts = []
    for out_dim, in_dim in shapes:
        s = math.sqrt(6.0 / (out_dim + in_dim))
        parts.append(rng.uniform(-s, s, size=out_dim * in_dim).astype(np.float32))
    return np.concatenate(parts).astype(np.float16)


def mlp_inputs(n: int, seed: int = 0):
    """Config 1: n rows of encoded inputs U(-1, 1) fp16 [32][n], sample records whose view
    directions are uniform on S^2 (z = 1 - 2u, phi = 2 pi v), and dL/d(output) fp16 [n][16]
    (channels 0-3 ~ N(0, 1), the rest zero)."""
    rng = np.random.default_rng(seed)
    x = rng.uniform(-1.0, 1.0, size=(32, n)).astype(np.float16)
    u, v = rng.random(n), rng.random(n)
    z = 1.0 - 2.0 * u
    r = np.sqrt(np.maximum(0.0, 1.0 - z * z))
    phi = 2.0 * math.pi * v
    d = np.stack([r * np.cos(phi), r * np.sin(phi), z], axis=1)
    coords = np.zeros((n, 7), np.float32)
    coords[:, :3] = rng.random((n, 3))
    coords[:, 3] = math.sqrt(3.0) / 1024.0
    coords[:, 4:7] = ((d + 1.0) * 0.5).astype(np.float32)
    dy = np.zeros((n, 16), np.float16)
    dy[:, :4] = rng.standard_normal((n, 4)).astype(np.float16)
    return x, coords, dy
