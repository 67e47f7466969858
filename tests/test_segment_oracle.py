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


def test_threaded_oracle_variants_match(oracle):
    """The threaded oracle paths the CPU baseline times give the single-threaded results."""
    vals = workloads.blob_grid_values(workloads.gaussian_blob_density())
    bits = np.packbits((vals > 0.01).reshape(-1, 8), axis=1, bitorder="little").reshape(-1)
    rays = workloads.march_rays_config2(3000, seed=4)
    a = oracle.march_rays(rays, bits, sample_limit=150000)
    b = oracle.march_rays_mt(rays, bits, 4, sample_limit=150000)
    assert a[2] == b[2] and (a[0] == b[0]).all() and a[1].tobytes() == b[1].tobytes()
    x, coords, dy = workloads.mlp_inputs(3000, seed=1)
    params = workloads.xavier_mlp_params(2)
    dx1, dw1 = oracle.mlp_backward(params, x, coords, dy)
    dx4, dw4 = oracle.mlp_backward(params, x, coords, dy, threads=4)
    assert dx1.tobytes() == dx4.tobytes()
    np.testing.assert_allclose(dw4, dw1, rtol=1e-12, atol=1e-12)
    rng = np.random.default_rng(0)
    n = 50000
    state = [rng.uniform(-1, 1, n).astype(np.float32), rng.uniform(-1, 1, n).astype(np.float16), rng.normal(size=n).astype(np.float32),
             np.zeros(n, np.float32), np.zeros(n, np.float32), np.zeros(n, np.uint32)]
    r1 = oracle.adam(10240, *state)
    r4 = oracle.adam(10240, *state, threads=4)
    assert all(p.tobytes() == q.tobytes() for p, q in zip(r1, r4))
