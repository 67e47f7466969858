"""Hash-grid layout and index: library vs oracle vs the reference's published layout numbers."""
from __future__ import annotations

import math

import numpy as np
import pytest


def test_reference_layout_matches_reference_totals(ngp):
    # ngp.train.h:44-86 at the reference config (8 levels x 4 features, T = 2^19):
    # 2,920,448 entries, 11,681,792 grid params, 11,692,032 params with the 10,240 MLP weights.
    lay = ngp.grid_layout()
    assert lay.n_entries == 2_920_448
    assert lay.n_params == 11_681_792
    assert lay.n_params + 10_240 == 11_692_032
    assert lay.level_resolutions() == [16 << l for l in range(8)]
    assert lay.level_scales() == [float((16 << l) - 1) for l in range(8)]
    assert lay.level_offsets() == [0, 4096, 36864, 299008, 823296, 1347584, 1871872, 2396160, 2920448]


def test_config0_layout(ngp):
    lay = ngp.config0_layout()
    assert lay.n_entries == 6_098_120 and lay.n_params == 12_196_240
    res = lay.level_resolutions()
    assert res[0] == 16 and res[-1] == 2048
    assert lay.level_scales()[0] == 15.0 and lay.level_scales()[-1] == 2047.0


@pytest.mark.parametrize("cfg", [(8, 4, 19, 16, 1.0), (16, 2, 19, 16, math.log2(128) / 15), (16, 2, 22, 16, math.log2(256) / 15),
                                 (4, 1, 12, 4, 0.5), (3, 8, 10, 2, 2.0)])
def test_layout_library_equals_oracle(ngp, oracle, cfg):
    lay = ngp.grid_layout(*cfg)
    offsets, res, scale = oracle.grid_layout(*cfg)
    assert lay.level_offsets() == offsets.tolist()
    assert lay.level_resolutions() == res.tolist()
    assert np.array(lay.level_scales(), np.float32).tobytes() == scale.tobytes()


def test_grid_index_dense_and_hash(oracle):
    # dense: x + y r + z r^2 while r^3 fits the level
    assert oracle.grid_index(4096, 16, 3, 5, 7) == 3 + 5 * 16 + 7 * 256
    # hashed: x ^ y*2654435761 ^ z*805459861 (mod 2^32), then % T
    x, y, z = 1234, 987, 4321
    h = (x ^ ((y * 2654435761) & 0xFFFFFFFF) ^ ((z * 805459861) & 0xFFFFFFFF)) % (1 << 19)
    assert oracle.grid_index(1 << 19, 2048, x, y, z) == h
    # resolution above 0x659 always hashes, even when the level is large
    assert oracle.grid_index(1 << 27, 0x65A, 1, 0, 0) == 1
    # corner at x == res aliases onto the next row exactly as the reference's arithmetic does
    assert oracle.grid_index(4096, 16, 16, 0, 0) == 16


def test_pcg32_published_vector(oracle):
    # pcg32_srandom_r(42, 54) from the PCG reference implementation's demo output
    u, _ = oracle.pcg32(42, 54, 0, 6)
    assert [hex(v) for v in u] == ["0xa15c02b7", "0x7b47f409", "0xba1d3330", "0x83d2f293", "0xbfa4784b", "0xcbed606e"]


def test_pcg32_advance_is_skip(oracle):
    u, f = oracle.pcg32(1337, 1, 0, 100)
    u2, f2 = oracle.pcg32(1337, 1, 37, 63)
    assert (u[37:] == u2).all() and (f[37:] == f2).all()
    assert ((f >= 0) & (f < 1)).all()

