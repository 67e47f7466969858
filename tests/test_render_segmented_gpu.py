"""Segmented evaluation marching (ngp_march_rays_segment + ngp_eval_composite_segment) against
the reference's flow (march every occupied step, then evaluate and composite), which
test_sampler_gpu pins to the reference kernels:

* every ray's samples over its segments are the single march's samples, bit for bit, also when
  a segment's sample limit leaves some listed rays for the next segment;
* the rendered image and its squared error are the single-pass ones, bit for bit (the error sum
  to 1e-12 relative: fp64 atomics in block order);
* the trainer's validate / test / render give the same results with segmented marching on or off.
"""
from __future__ import annotations

import math

import numpy as np
import pytest

import workloads

pytestmark = pytest.mark.gpu


def T(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.fixture(scope="module")
def blob_bitfield():
    vals = workloads.blob_grid_values(workloads.gaussian_blob_density())
    return np.packbits((vals > 0.01).reshape(-1, 8), axis=1, bitorder="little").reshape(-1)


@pytest.fixture(scope="module")
def small_scene():
    return workloads.procedural_dataset(n_train=6, n_test=2, width=96, height=80, seed=5)


def _full_march(ngp, rays, bits, limit=1 << 22):
    import torch

    n = rays.shape[0]
    coords = torch.zeros((limit, 7), dtype=torch.float32, device="cuda")
    ns = torch.zeros((n, 2), dtype=torch.int32, device="cuda")
    msc = torch.zeros(ngp.march_scratch_words(n), dtype=torch.int32, device="cuda")
    sc = torch.zeros(1, dtype=torch.int32, device="cuda")
    ngp.march_rays(rays, bits, coords, ns, msc, sc, sample_limit=limit)
    torch.cuda.synchronize()
    return ns.cpu().numpy().view(np.uint32), coords.cpu().numpy()


def _segment_march_python(ngp, rays, bits, caps, limits):
    """Drives the segment march with the per-ray bookkeeping done on the host; returns each ray's
    records over all its segments and the segment count that a partial (prefix) fit occurred in."""
    import torch

    n = rays.shape[0]
    coords = torch.zeros((max(limits), 7), dtype=torch.float32, device="cuda")
    ns = torch.zeros((n, 2), dtype=torch.int32, device="cuda")
    t_out = torch.zeros(n, dtype=torch.float32, device="cuda")
    msc = torch.zeros(ngp.march_scratch_words(n), dtype=torch.int32, device="cuda")
    counters = torch.zeros(4, dtype=torch.int32, device="cuda")
    t_state = torch.zeros(n, dtype=torch.float32, device="cuda")
    marched = torch.zeros(n, dtype=torch.int32, device="cuda")
    per_ray = [[] for _ in range(n)]
    todo = np.arange(n, dtype=np.int32)
    partial = 0
    seg = 0
    while todo.size:
        cap, limit = caps[min(seg, len(caps) - 1)], limits[min(seg, len(limits) - 1)]
        lst = None if seg == 0 else T(todo)
        ngp.march_rays_segment(rays, bits, coords, ns, t_out, msc, counters, cap, max_entries=int(todo.size), ray_list=lst,
                               t_state=None if seg == 0 else t_state, marched=None if seg == 0 else marched, sample_limit=limit)
        torch.cuda.synchronize()
        c = counters.cpu().numpy().view(np.uint32)
        complete = int(c[1])
        assert 0 < complete <= todo.size
        partial += complete < todo.size
        nsh = ns.cpu().numpy().view(np.uint32)[: todo.size]
        to = t_out.cpu().numpy()[: todo.size]
        co = coords.cpu().numpy()
        ts, mk = t_state.cpu().numpy(), marched.cpu().numpy()
        assert (nsh[complete:, 0] == 0).all()
        assert int(nsh[:complete, 0].sum()) <= limit
        nxt = []
        for k in range(todo.size):
            i = int(todo[k])
            if k >= complete:
                nxt.append(i)
                continue
            cnt, base = int(nsh[k, 0]), int(nsh[k, 1])
            if cnt:
                per_ray[i].append(co[base:base + cnt])
            assert cnt <= cap
            if to[k] >= 0.0:
                assert cnt == cap  # only a ray stopped by the cap continues
                ts[i], mk[i] = to[k], mk[i] + cnt
                nxt.append(i)
        t_state.copy_(torch.from_numpy(ts))
        marched.copy_(torch.from_numpy(mk))
        todo = np.asarray(nxt, dtype=np.int32)
        seg += 1
        assert seg < 200
    return per_ray, partial


@pytest.mark.parametrize("density,later_limit", [(None, 9000), (0.3, 150000)])
def test_segments_concatenate_to_the_full_march(ngp, blob_bitfield, density, later_limit):
    if density is None:
        bits = blob_bitfield
    else:
        occ = np.random.default_rng(5).random(128 ** 3) < density
        bits = np.packbits(occ.reshape(-1, 8), axis=1, bitorder="little").reshape(-1)
    n = 4096
    rays = T(workloads.march_rays_config2(n, seed=21))
    bits = T(bits)
    full_ns, full_coords = _full_march(ngp, rays, bits)
    # caps 7 then 40 then the rest; later segments with a limit small enough to split the list
    per_ray, partial = _segment_march_python(ngp, rays, bits, caps=[7, 40, 1024], limits=[7 * n, later_limit])
    assert partial > 0
    for i in range(n):
        cnt, base = int(full_ns[i, 0]), int(full_ns[i, 1])
        got = np.concatenate(per_ray[i]) if per_ray[i] else np.zeros((0, 7), np.float32)
        assert got.shape[0] == cnt, i
        assert got.tobytes() == full_coords[base:base + cnt].tobytes(), i


def test_first_segment_must_fit(ngp, blob_bitfield):
    import torch

    n = 1000
    rays = T(workloads.march_rays_config2(n, seed=3))
    z = torch.zeros(ngp.march_scratch_words(n), dtype=torch.int32, device="cuda")
    with pytest.raises(RuntimeError, match="first segment"):
        ngp.march_rays_segment(rays, T(blob_bitfield), torch.zeros((4096, 7), device="cuda"), torch.zeros((n, 2), dtype=torch.int32, device="cuda"),
                               torch.zeros(n, device="cuda"), z, torch.zeros(4, dtype=torch.int32, device="cuda"), 64, sample_limit=4096)


def _network(ngp):
    layout = ngp.grid_layout(16, 2, 19, 16, math.log2(128.0) / 15.0)
    _, table, _ = workloads.encode_inputs(1, layout.n_params, 16, 2, seed=4)
    table = (table.astype(np.float32) * 2e4).astype(np.float16)
    mlp = workloads.xavier_mlp_params(9)
    mlp[2048:2048 + 64] = np.random.default_rng(3).uniform(0.2, 0.5, 64).astype(np.float16)
    return layout, T(np.concatenate([mlp, table]).view(np.int16))


def test_segmented_render_matches_single_pass(ngp, small_scene, blob_bitfield):
    import torch

    tr = small_scene["train"]
    pix, cam = T(tr["pixels"]), T(tr["camera"])
    F, H, W = tr["pixels"].shape[:3]
    (fx, fy), (cx, cy) = tr["focal"], tr["principal"]
    layout, params = _network(ngp)
    bits = T(blob_bitfield)
    n = W * H
    rays = torch.zeros((n, 6), dtype=torch.float32, device="cuda")
    ngp.make_eval_rays(cam, 1, W, H, fx, fy, cx, cy, 0, n, rays)
    limit = 1 << 21
    scratch = torch.zeros(ngp.loss_scratch_bytes(n), dtype=torch.uint8, device="cuda")

    # single pass: march everything, evaluate in front of the stopping points, composite
    ns, coords = (torch.zeros((n, 2), dtype=torch.int32, device="cuda"), torch.zeros((limit, 7), dtype=torch.float32, device="cuda"))
    msc = torch.zeros(ngp.march_scratch_words(n), dtype=torch.int32, device="cuda")
    sc = torch.zeros(1, dtype=torch.int32, device="cuda")
    ngp.march_rays(rays, bits, coords, ns, msc, sc, sample_limit=limit)
    torch.cuda.synchronize()
    m = (max(int(sc.item()), 6 * n) + 127) // 128 * 128
    enc = torch.zeros((32, m), dtype=torch.float16, device="cuda")
    out = torch.zeros((m, 16), dtype=torch.float16, device="cuda")
    rows = torch.zeros(m, dtype=torch.int32, device="cuda")
    ngp.eval_network_progressive(n, layout, params, coords, m, ns, enc, out, rows, scratch)
    img_a = torch.zeros((n, 3), dtype=torch.float32, device="cuda")
    sse_a = torch.zeros(1, dtype=torch.float64, device="cuda")
    cmp_a = torch.zeros((H, 2 * W, 3), dtype=torch.uint8, device="cuda")
    ngp.eval_composite(n, 0, 1, W, H, pix, ns, coords, out, sse=sse_a, comparison=cmp_a, rendered=img_a)

    # segmented: caps 6, 24, rest; later segments with a small sample limit (lists split)
    img_b = torch.zeros((n, 3), dtype=torch.float32, device="cuda")
    sse_b = torch.zeros(1, dtype=torch.float64, device="cuda")
    cmp_b = torch.zeros((H, 2 * W, 3), dtype=torch.uint8, device="cuda")
    caps, limits = [6, 24, 1024], [6 * n, 20000]
    t_out = torch.zeros(n, dtype=torch.float32, device="cuda")
    t_state = torch.zeros(n, dtype=torch.float32, device="cuda")
    marched = torch.zeros(n, dtype=torch.int32, device="cuda")
    state = torch.zeros((n, 4), dtype=torch.float32, device="cuda")
    lists = torch.zeros((2, n), dtype=torch.int32, device="cuda")
    counters = torch.zeros(4, dtype=torch.int32, device="cuda")
    max_entries, seg, partial = n, 0, 0
    while True:
        first = seg == 0
        lst = None if first else lists[(seg - 1) & 1]
        n_dev = None if first else counters[2 + ((seg - 1) & 1):3 + ((seg - 1) & 1)]
        ngp.march_rays_segment(rays, bits, coords, ns, t_out, msc, counters, caps[min(seg, 2)], max_entries=max_entries, n_entries=n_dev,
                               ray_list=lst, t_state=None if first else t_state, marched=None if first else marched,
                               sample_limit=limits[min(seg, 1)])
        torch.cuda.synchronize()
        c = counters.cpu().numpy().view(np.uint32)
        complete = int(c[1])
        if complete == 0:
            break
        n_in = n if first else int(c[2 + ((seg - 1) & 1)])
        partial += complete < n_in
        used = min(int(c[0]), limits[min(seg, 1)])
        if used:
            mm = (used + 127) // 128 * 128
            ngp.eval_network_progressive(complete, layout, params, coords, mm, ns, enc, out, rows, scratch, enc_stride=mm)
        counters[2 + (seg & 1)] = 0
        ngp.eval_composite_segment(max_entries, counters[1:2], ns, coords, out, t_out, t_state, marched, state, lists[seg & 1],
                                   counters[2 + (seg & 1):3 + (seg & 1)], 0, 1, W, H, n_entries=n_dev, ray_list=lst, pixels=pix, sse=sse_b,
                                   comparison=cmp_b, rendered=img_b)
        if not first:
            max_entries = n_in
        seg += 1
        assert seg < 64
    torch.cuda.synchronize()
    assert seg >= 3 and partial > 0
    assert img_a.cpu().numpy().tobytes() == img_b.cpu().numpy().tobytes()
    assert cmp_a.cpu().numpy().tobytes() == cmp_b.cpu().numpy().tobytes()
    a, b = float(sse_a.item()), float(sse_b.item())
    assert a > 0 and abs(a - b) <= 1e-12 * a


def test_trainer_segmented_eval_identical(ngp):
    import torch

    scene = workloads.procedural_dataset(n_train=8, n_test=2, n_validation=1, width=160, height=120, seed=13, device="cuda")
    m = ngp.InstantNGP(scene)
    m.train(150)
    cam = scene["test"]["camera"][1]
    f, p = scene["test"]["focal"], scene["test"]["principal"]
    results = {}
    for seg in (False, True):
        m.set_segmented_eval(seg)
        rgb = m.render(cam, 160, 120, f, p)
        torch.cuda.synchronize()
        t = m.test(1, with_images=True)
        v = m.validate()
        results[seg] = (rgb.cpu().numpy().tobytes(), t["images"][0].tobytes(), t["mse"], v["mse"])
    m.close()
    a, b = results[False], results[True]
    assert a[0] == b[0] and a[1] == b[1]
    assert abs(a[2] - b[2]) <= 1e-12 * a[2] and abs(a[3] - b[3]) <= 1e-12 * a[3]


def test_segment_outputs_match_oracle(ngp, oracle):
    """Per segment, the library's counts, records and continuation t equal the oracle's
    restatement bit for bit (first segment, then a listed continuation segment)."""
    import torch

    occ = np.random.default_rng(7).random(128 ** 3) < 0.3
    bits_h = np.packbits(occ.reshape(-1, 8), axis=1, bitorder="little").reshape(-1)
    n, cap0, cap1 = 2048, 9, 40
    rays_h = workloads.march_rays_config2(n, seed=23)
    rays, bits = T(rays_h), T(bits_h)
    coords = torch.zeros((n * cap1, 7), dtype=torch.float32, device="cuda")
    ns = torch.zeros((n, 2), dtype=torch.int32, device="cuda")
    t_out = torch.zeros(n, dtype=torch.float32, device="cuda")
    msc = torch.zeros(ngp.march_scratch_words(n), dtype=torch.int32, device="cuda")
    counters = torch.zeros(4, dtype=torch.int32, device="cuda")
    ngp.march_rays_segment(rays, bits, coords, ns, t_out, msc, counters, cap0, sample_limit=n * cap1)
    torch.cuda.synchronize()
    ons, ocoords, ot = oracle.march_segment(rays_h, bits_h, cap0)
    g_ns = ns.cpu().numpy().view(np.uint32)
    assert (g_ns == ons).all() and int(counters[1].item()) == n
    assert coords.cpu().numpy()[: ocoords.shape[0]].tobytes() == ocoords.tobytes()
    g_t = t_out.cpu().numpy()
    assert g_t.tobytes() == ot.tobytes()
    # continuation of the rays the cap stopped, listed in reverse order
    lst = np.nonzero(ot >= 0.0)[0][::-1].astype(np.uint32)
    assert lst.size > 100
    t_state = np.zeros(n, np.float32)
    t_state[lst] = ot[lst]
    marched = np.zeros(n, np.uint32)
    marched[lst] = cap0
    ngp.march_rays_segment(rays, bits, coords, ns, t_out, msc, counters, cap1, max_entries=int(lst.size), ray_list=T(lst.view(np.int32)),
                           t_state=T(t_state), marched=T(marched.view(np.int32)), sample_limit=n * cap1)
    torch.cuda.synchronize()
    ons, ocoords, ot2 = oracle.march_segment(rays_h, bits_h, cap1, ray_list=lst, t_state=t_state, marched=marched)
    assert (ns.cpu().numpy().view(np.uint32)[: lst.size] == ons).all()
    assert coords.cpu().numpy()[: ocoords.shape[0]].tobytes() == ocoords.tobytes()
    assert t_out.cpu().numpy()[: lst.size].tobytes() == ot2.tobytes()


@pytest.mark.parametrize("ranks", [1, 3, 4])
def test_tile_partitioned_render_assembles_the_image(ngp, ranks):
    """Inference partitioned by 64 x 64 tiles (rank r of N renders tiles r, r + N, ...; the tile
    loop of run_evaluation, ngp.train.cu:1616-1620): the ranks' tiles, rendered one after another
    on this GPU, fill the image exactly once and give the whole-image render bit for bit,
    including the clipped tiles at the right and bottom edges (200 x 150 is not a multiple of 64)."""
    import torch

    scene = workloads.procedural_dataset(n_train=8, n_test=1, width=200, height=150, seed=17, device="cuda")
    m = ngp.InstantNGP(scene)
    m.train(100)
    cam = scene["test"]["camera"][0]
    f, p = scene["test"]["focal"], scene["test"]["principal"]
    full = m.render(cam, 200, 150, f, p)
    tiled = torch.full((200 * 150, 3), -1.0, dtype=torch.float32, device="cuda")
    for r in range(ranks):
        m.render_tiles(cam, 200, 150, f, p, r, ranks, tiled)
    torch.cuda.synchronize()
    m.close()
    assert (tiled >= 0).all()
    assert tiled.cpu().numpy().tobytes() == full.cpu().numpy().tobytes()
