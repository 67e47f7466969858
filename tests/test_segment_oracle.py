"""CPU tier: segmented marching (the evaluation march resumed where the previous segment stopped)
restated in the oracle gives each ray the samples of one uninterrupted march, bit for bit --
against the reference kernel's own golden output and against the oracle's single march on a
scattered occupancy grid.  The GPU segment march is checked against the same single march in
test_render_segmented_gpu.py.  No GPU needed."""
from __future__ import annotations

import numpy as np
import pytest

import workloads
from conftest import GOLDEN


def segmented(oracle, rays, bits, caps):
    """Each ray's records over its segments (host bookkeeping of t_state / marched)."""
    n = rays.shape[0]
    per_ray = [[] for _ in range(n)]
    t_state = np.zeros(n, np.float32)
    marched = np.zeros(n, np.uint32)
    todo = None
    seg = 0
    while todo is None or todo.size:
        cap = caps[min(seg, len(caps) - 1)]
        ns, coords, t_out = oracle.march_segment(rays, bits, cap, ray_list=todo, t_state=None if seg == 0 else t_state,
                                                 marched=None if seg == 0 else marched)
        ids = np.arange(n, dtype=np.uint32) if todo is None else todo
        nxt = []
        for k, i in enumerate(ids):
            cnt, base = int(ns[k, 0]), int(ns[k, 1])
            assert cnt <= cap
            if cnt:
                per_ray[i].append(coords[base:base + cnt])
            if t_out[k] >= 0.0:
                assert cnt == cap
                t_state[i] = t_out[k]
                marched[i] += cnt
                nxt.append(i)
        todo = np.asarray(nxt, np.uint32)
        seg += 1
        assert seg < 300
    return per_ray, seg


def check(per_ray, numsteps, coords):
    for i, parts in enumerate(per_ray):
        cnt, base = int(numsteps[i, 0]), int(numsteps[i, 1])
        got = np.concatenate(parts) if parts else np.zeros((0, 7), np.float32)
        assert got.shape[0] == cnt, i
        assert got.tobytes() == coords[base:base + cnt].tobytes(), i


def test_segments_match_reference_golden(oracle):
    p = GOLDEN / "march_ref.npz"
    if not p.exists():
        pytest.skip("march_ref.npz not generated yet")
    g = np.load(p)
    vals = workloads.blob_grid_values(workloads.gaussian_blob_density())
    bits = np.packbits((vals > 0.01).reshape(-1, 8), axis=1, bitorder="little").reshape(-1)
    rays = workloads.march_rays_config2(int(g["n"]), seed=int(g["seed"]))
    per_ray, segs = segmented(oracle, rays, bits, caps=[5, 30, 1024])
    assert segs >= 3
    counts = g["numsteps"].astype(np.uint32)
    bases = np.concatenate([[0], np.cumsum(counts)[:-1]]).astype(np.uint32)
    check(per_ray, np.stack([counts, bases], axis=1), g["coords"])


@pytest.mark.parametrize("caps", [[1, 1024], [3, 17, 64], [64, 128, 1024]])
def test_segments_match_single_march_scattered_grid(oracle, caps):
    occ = np.random.default_rng(7).random(128 ** 3) < 0.3
    bits = np.packbits(occ.reshape(-1, 8), axis=1, bitorder="little").reshape(-1)
    rays = workloads.march_rays_config2(512, seed=19)
    ns, coords, total = oracle.march_rays(rays, bits)
    assert total > 512 * 64  # long rays: several segments each
    per_ray, _ = segmented(oracle, rays, bits, caps)
    check(per_ray, ns, coords)
