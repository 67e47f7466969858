"""Occupancy grid, ray marching, compositing/loss and Adam: CUDA library vs the CPU oracle and the
reference's own kernels (oracle/_ref).

Bars (north_star: occupancy bitfield, per-ray sample counts and positions bit-exact):
* marching, library vs oracle and vs the reference kernels: per-ray counts and sample records
  bit-exact (the reference places rays in atomic order; rays are matched by their index);
* grid samples and EMA: bit-exact; bitfield: bit-exact except cells within 1e-6 relative of the
  threshold (the reference's mean is an order-dependent float atomic sum);
* loss / gradients (fp32 with libm transcendental functions): per-ray loss within 1e-5 relative,
  compacted counts exact, fp16 gradients within 2 ulp;
* Adam: within 1e-6 relative of the oracle.
"""
from __future__ import annotations

import ctypes
import math

import numpy as np
import pytest

import workloads

pytestmark = pytest.mark.gpu

V = ctypes.c_void_p


def T(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def P(t):
    return V(t.data_ptr())


@pytest.fixture(scope="module")
def blob_bitfield():
    vals = workloads.blob_grid_values(workloads.gaussian_blob_density())
    bits = np.packbits((vals > 0.01).reshape(-1, 8), axis=1, bitorder="little").reshape(-1)
    return bits


@pytest.fixture(scope="module")
def small_scene():
    return workloads.procedural_dataset(n_train=6, n_test=2, width=96, height=80, seed=5)


def run_march(ngp, rays, bits, jitter, step=0, limit=1 << 22):
    import torch

    n = rays.shape[0]
    coords = torch.zeros((limit, 7), dtype=torch.float32, device="cuda")
    numsteps = torch.zeros((n, 2), dtype=torch.int32, device="cuda")
    totals = torch.zeros(ngp.march_scratch_words(n), dtype=torch.int32, device="cuda")
    counter = torch.zeros(1, dtype=torch.int32, device="cuda")
    ngp.march_rays(T(rays), T(bits), coords, numsteps, totals, counter, sample_limit=limit, jitter=jitter, step=step)
    torch.cuda.synchronize()
    return numsteps.cpu().numpy().view(np.uint32), coords.cpu().numpy(), int(counter.item())


@pytest.mark.parametrize("n", [1, 127, 4096])
@pytest.mark.parametrize("jitter", [False, True])
def test_march_bit_exact_vs_oracle(ngp, oracle, blob_bitfield, n, jitter):
    rays = workloads.march_rays_config2(n, seed=n)
    ns, coords, total = run_march(ngp, rays, blob_bitfield, jitter, step=7)
    ons, ocoords, ototal = oracle.march_rays(rays, blob_bitfield, jitter=jitter, step=7)
    assert total == ototal
    assert (ns == ons).all()
    used = int(ns[:, 0].sum())
    assert coords[:used].tobytes() == ocoords[:used].tobytes()


@pytest.mark.parametrize("density", [0.02, 0.3, 0.9])
def test_march_random_bitfield_runs(ngp, oracle, density):
    """Scattered occupancy: rays cross many separate occupied runs (beyond the per-ray run
    record, which makes those rays march a second time) -- still bit-exact."""
    rng = np.random.default_rng(int(density * 100))
    occ = rng.random(128 ** 3) < density
    bits = np.packbits(occ.reshape(-1, 8), axis=1, bitorder="little").reshape(-1)
    rays = workloads.march_rays_config2(4096, seed=11)
    ns, coords, total = run_march(ngp, rays, bits, True, step=3)
    ons, ocoords, ototal = oracle.march_rays(rays, bits, jitter=True, step=3)
    assert total == ototal and (ns == ons).all()
    used = int(ns[:, 0].sum())
    assert used > 0
    assert coords[:used].tobytes() == ocoords[:used].tobytes()


def test_march_full_config2(ngp, oracle, blob_bitfield):
    """Config 2 at full size: 2^18 rays, bit-exact against the oracle."""
    rays = workloads.march_rays_config2(1 << 18, seed=2)
    ns, coords, total = run_march(ngp, rays, blob_bitfield, False)
    ons, ocoords, ototal = oracle.march_rays(rays, blob_bitfield)
    assert total == ototal and (ns == ons).all()
    used = int(ns[:, 0].sum())
    assert used > 100000
    assert coords[:used].tobytes() == ocoords[:used].tobytes()


def test_march_sample_limit_drops_whole_rays(ngp, oracle, blob_bitfield):
    rays = workloads.march_rays_config2(2048, seed=9)
    ns, _, total = run_march(ngp, rays, blob_bitfield, False, limit=20000)
    ons, _, _ = oracle.march_rays(rays, blob_bitfield, sample_limit=20000)
    assert (ns == ons).all() and total > 20000
    assert ns[:, 0].sum() <= 20000


def test_march_empty_grid(ngp, blob_bitfield):
    rays = workloads.march_rays_config2(300, seed=1)
    ns, _, total = run_march(ngp, rays, np.zeros_like(blob_bitfield), True)
    assert total == 0 and (ns == 0).all()


def _scene_tensors(scene):
    tr = scene["train"]
    return T(tr["pixels"]), T(tr["camera"]), tr


def test_training_rays_vs_reference_kernel(ngp, reflib, small_scene, blob_bitfield):
    """generate_training_samples_kernel vs ours: per ray, the same sample count and records."""
    import torch

    pix, cam, tr = _scene_tensors(small_scene)
    F, H, W = tr["pixels"].shape[:3]
    bits = T(blob_bitfield)
    n, limit, step = 8192, 1 << 22, 3
    (fx, fy), (cx, cy) = tr["focal"], tr["principal"]
    # reference
    rc = torch.zeros(1, dtype=torch.int32, device="cuda")
    sc = torch.zeros(1, dtype=torch.int32, device="cuda")
    r_idx = torch.zeros(n, dtype=torch.int32, device="cuda")
    r_rays = torch.zeros((n, 6), dtype=torch.float32, device="cuda")
    r_ns = torch.zeros((n, 2), dtype=torch.int32, device="cuda")
    r_coords = torch.zeros((limit, 7), dtype=torch.float32, device="cuda")
    reflib.call("ref_generate_training_samples", ctypes.c_uint32(n), ctypes.c_uint32(limit), ctypes.c_uint32(step), ctypes.c_uint32(F),
                ctypes.c_uint32(W), ctypes.c_uint32(H), ctypes.c_float(fx), ctypes.c_float(fy), ctypes.c_float(cx), ctypes.c_float(cy), P(cam),
                P(bits), P(rc), P(sc), P(r_idx), P(r_rays), P(r_ns), P(r_coords))
    # ours
    o_ns = torch.zeros((n, 2), dtype=torch.int32, device="cuda")
    o_rays = torch.zeros((n, 6), dtype=torch.float32, device="cuda")
    o_idx = torch.zeros(n, dtype=torch.int32, device="cuda")
    o_coords = torch.zeros((limit, 7), dtype=torch.float32, device="cuda")
    totals = torch.zeros(ngp.march_scratch_words(n), dtype=torch.int32, device="cuda")
    orc = torch.zeros(1, dtype=torch.int32, device="cuda")
    osc = torch.zeros(1, dtype=torch.int32, device="cuda")
    ngp.march_training_rays(cam, F, W, H, fx, fy, cx, cy, step, n, limit, bits, o_coords, o_rays, o_idx, o_ns, totals, orc, osc)
    torch.cuda.synchronize()
    assert int(sc.item()) == int(osc.item())
    k = int(rc.item())
    ridx = r_idx[:k].cpu().numpy()
    rns = r_ns[:k].cpu().numpy()
    rco = r_coords.cpu().numpy()
    ons = o_ns.cpu().numpy()
    oco = o_coords.cpu().numpy()
    orays = o_rays.cpu().numpy()
    rrays = r_rays[:k].cpu().numpy()
    assert k == int((ons[:, 0] > 0).sum())
    assert (ons[ridx, 0] == rns[:, 0]).all()
    assert orays[ridx].tobytes() == rrays.tobytes()
    for j in range(k):
        a = rco[rns[j, 1]: rns[j, 1] + rns[j, 0]]
        b = oco[ons[ridx[j], 1]: ons[ridx[j], 1] + rns[j, 0]]
        assert a.tobytes() == b.tobytes(), j


def test_eval_rays_vs_reference_kernel(ngp, reflib, small_scene, blob_bitfield):
    """generate_evaluation_samples_kernel vs ours on one 4096-pixel tile: per pixel, the same samples."""
    import torch

    pix, cam, tr = _scene_tensors(small_scene)
    F, H, W = tr["pixels"].shape[:3]
    bits = T(blob_bitfield)
    n, off, image = 4096, 1000, 1
    (fx, fy), (cx, cy) = tr["focal"], tr["principal"]
    sc = torch.zeros(1, dtype=torch.int32, device="cuda")
    ov = torch.zeros(1, dtype=torch.int32, device="cuda")
    r_ns = torch.zeros((n, 2), dtype=torch.int32, device="cuda")
    r_coords = torch.zeros((n * 1024, 7), dtype=torch.float32, device="cuda")
    reflib.call("ref_generate_evaluation_samples", ctypes.c_uint32(n), ctypes.c_uint32(off), ctypes.c_uint32(n * 1024), ctypes.c_uint32(W),
                ctypes.c_uint32(H), ctypes.c_float(fx), ctypes.c_float(fy), ctypes.c_float(cx), ctypes.c_float(cy), P(cam), ctypes.c_uint32(image),
                P(bits), P(sc), P(ov), P(r_ns), P(r_coords))
    rays = torch.zeros((n, 6), dtype=torch.float32, device="cuda")
    ngp.make_eval_rays(cam, image, W, H, fx, fy, cx, cy, off, n, rays)
    torch.cuda.synchronize()
    ns, coords, total = run_march(ngp, rays.cpu().numpy(), blob_bitfield, False)
    rns = r_ns.cpu().numpy()
    rco = r_coords.cpu().numpy()
    assert total == int(sc.item()) and int(ov.item()) == 0
    assert (ns[:, 0] == rns[:, 0]).all()
    for i in np.nonzero(rns[:, 0])[0]:
        assert rco[rns[i, 1]: rns[i, 1] + rns[i, 0]].tobytes() == coords[ns[i, 1]: ns[i, 1] + ns[i, 0]].tobytes(), i


def test_grid_samples_and_update_vs_reference(ngp, oracle, reflib):
    import torch

    vals0 = workloads.blob_grid_values(workloads.gaussian_blob_density())
    vals0[::97] = -1.0  # some untrained cells
    nu, nn = 1 << 16, 1 << 16
    values = T(vals0)
    coords = torch.zeros((nu + nn, 7), dtype=torch.float32, device="cuda")
    idx = torch.zeros(nu + nn, dtype=torch.int32, device="cuda")
    ngp.density_grid_samples(nu, nn, 5, values, coords, idx)
    rcoords = torch.zeros_like(coords)
    ridx = torch.zeros_like(idx)
    reflib.call("ref_grid_samples", ctypes.c_uint32(nu), ctypes.c_uint32(nn), ctypes.c_uint32(5), P(values), P(rcoords), P(ridx))
    torch.cuda.synchronize()
    oc, oi = oracle.grid_samples(nu, nn, 5, vals0)
    assert coords.cpu().numpy().tobytes() == rcoords.cpu().numpy().tobytes() == oc.tobytes()
    assert (idx.cpu().numpy().view(np.uint32) == oi).all() and (ridx.cpu().numpy().view(np.uint32) == oi).all()

    # splat + EMA + mean + bitfield on the same densities
    rng = np.random.default_rng(4)
    dens = rng.normal(-1.0, 2.0, nu + nn).astype(np.float16)
    D = T(dens)
    scratch = torch.zeros(128 ** 3, dtype=torch.float32, device="cuda")
    ngp.density_grid_splat(nu + nn, idx, D, scratch)
    torch.cuda.synchronize()
    splatted = scratch.cpu().numpy()
    v_ours = values.clone()
    partial = torch.zeros(ngp.density_grid_partials(), dtype=torch.float32, device="cuda")
    mean = torch.zeros(1, dtype=torch.float32, device="cuda")
    bits = torch.zeros(128 ** 3 // 8, dtype=torch.uint8, device="cuda")
    occ = torch.zeros(1, dtype=torch.int32, device="cuda")
    ngp.density_grid_update(v_ours, scratch, partial, mean, bits, occ)
    v_ref = values.clone()
    rs = torch.zeros_like(scratch)
    rmean = torch.zeros(1, dtype=torch.float32, device="cuda")
    rbits = torch.zeros_like(bits)
    rocc = torch.zeros_like(occ)
    reflib.call("ref_grid_update", ctypes.c_uint32(nu + nn), P(idx), P(D), P(rs), P(v_ref), P(rmean), P(rbits), P(rocc))
    torch.cuda.synchronize()
    assert (scratch == 0).all()  # cleared for the next update
    assert v_ours.cpu().numpy().tobytes() == v_ref.cpu().numpy().tobytes()
    ov, omean, obits, ocnt = oracle.grid_update(vals0, splatted)
    assert v_ours.cpu().numpy().tobytes() == ov.tobytes()
    m = float(mean.item())
    assert abs(m - omean) <= 1e-5 * omean and abs(m - float(rmean.item())) <= 1e-5 * omean
    thr = min(0.01, m)
    near = np.abs(ov - thr) <= 1e-6 * thr
    ours_bits = np.unpackbits(bits.cpu().numpy(), bitorder="little").astype(bool)
    ref_bits = np.unpackbits(rbits.cpu().numpy(), bitorder="little").astype(bool)
    ora_bits = np.unpackbits(obits, bitorder="little").astype(bool)
    assert (ours_bits[~near] == ref_bits[~near]).all() and (ours_bits[~near] == ora_bits[~near]).all()
    assert int(occ.item()) == int(ours_bits.sum())


def test_mark_untrained_vs_reference(ngp, reflib, small_scene):
    import torch

    pix, cam, tr = _scene_tensors(small_scene)
    F, H, W = tr["pixels"].shape[:3]
    (fx, fy), (cx, cy) = tr["focal"], tr["principal"]
    ours = torch.zeros(128 ** 3, dtype=torch.float32, device="cuda")
    ref = torch.zeros_like(ours)
    ngp.density_grid_mark_untrained(cam, F, W, H, fx, fy, cx, cy, ours)
    reflib.call("ref_mark_untrained", P(ref), ctypes.c_uint32(F), ctypes.c_uint32(W), ctypes.c_uint32(H), ctypes.c_float(fx), ctypes.c_float(fy),
                ctypes.c_float(cx), ctypes.c_float(cy), P(cam))
    torch.cuda.synchronize()
    a, b = ours.cpu().numpy(), ref.cpu().numpy()
    assert 0.0 < (a == 0).mean() < 1.0
    assert (a != b).mean() < 1e-4  # cells decided by a last-ulp comparison may differ


def test_adam_vs_oracle(ngp, oracle):
    import torch

    rng = np.random.default_rng(0)
    n, n_mlp = 40000, 10240
    master = rng.uniform(-0.1, 0.1, n).astype(np.float32)
    grads = rng.normal(0, 10, n).astype(np.float32)
    grads[n_mlp::3] = 0.0  # sparse grid entries are skipped
    m = rng.normal(0, 0.01, n).astype(np.float32)
    v = rng.uniform(0, 0.01, n).astype(np.float32)
    steps = rng.integers(0, 5, n).astype(np.uint32)
    params = master.astype(np.float16)
    tm, tp, tg, tmm, tv, ts = (T(a) for a in (master, params.view(np.int16), grads, m, v, steps.view(np.int32)))
    ngp.adam_step(n_mlp, tm, tp, tg, tmm, tv, ts)
    torch.cuda.synchronize()
    om, op, omm, ov, os_ = oracle.adam(n_mlp, master, params, grads, m, v, steps)
    np.testing.assert_allclose(tm.cpu().numpy(), om, rtol=1e-6, atol=1e-9)
    np.testing.assert_allclose(tmm.cpu().numpy(), omm, rtol=1e-6, atol=1e-12)
    np.testing.assert_allclose(tv.cpu().numpy(), ov, rtol=1e-6, atol=1e-12)
    assert (ts.cpu().numpy().view(np.uint32) == os_).all()
    g = tg.cpu().numpy()
    assert (g[n_mlp:] == 0).all() and (g[:n_mlp] == grads[:n_mlp]).all()  # grid gradient cleared, MLP kept


def test_adam_rate_table_bit_identical(ngp):
    """Adam with the per-step-count rate table (partly covering the step counts, the rest
    computed) gives the same bits as Adam computing every rate."""
    import torch

    rng = np.random.default_rng(5)
    n, n_mlp = 50000, 10240
    master = rng.uniform(-0.1, 0.1, n).astype(np.float32)
    grads = rng.normal(0, 10, n).astype(np.float32)
    grads[n_mlp::4] = 0.0
    m = rng.normal(0, 0.01, n).astype(np.float32)
    v = rng.uniform(0, 0.01, n).astype(np.float32)
    steps = rng.integers(0, 3000, n).astype(np.uint32)
    params = master.astype(np.float16)
    a = [T(x) for x in (master, params.view(np.int16), grads, m, v, steps.view(np.int32))]
    b = [x.clone() for x in a]
    table = torch.zeros(4096, dtype=torch.float32, device="cuda")
    ngp.adam_lr_table(table, 1, 1000)
    ngp.adam_lr_table(table, 1001, 1000)
    ngp.adam_step(n_mlp, *a)
    ngp.adam_step_table(n_mlp, *b, table, 2000)
    torch.cuda.synchronize()
    for x, y in zip(a, b):
        assert x.cpu().numpy().tobytes() == y.cpu().numpy().tobytes()


def test_adam_vs_reference_kernel(ngp, reflib):
    """The reference's adam_step_kernel on fp16 gradients vs ours on the same values in fp32."""
    import torch

    total = int(reflib.lib.ref_total_param_count())
    n_mlp = int(reflib.lib.ref_mlp_param_count())
    rng = np.random.default_rng(1)
    master = rng.uniform(-0.1, 0.1, total).astype(np.float32)
    g16 = rng.normal(0, 5, total).astype(np.float16)
    g16[n_mlp::2] = 0
    params = master.astype(np.float16)
    zeros = np.zeros(total, np.float32)
    r = [T(a) for a in (master, params.view(np.int16), g16.view(np.int16), zeros, zeros, np.zeros(total, np.int32))]
    o = [T(a) for a in (master, params.view(np.int16), g16.astype(np.float32), zeros, zeros, np.zeros(total, np.int32))]
    for _ in range(3):
        reflib.call("ref_adam", P(r[0]), P(r[1]), P(r[2]), P(r[3]), P(r[4]), P(r[5]))
        ngp.adam_step(n_mlp, o[0], o[1], o[2], o[3], o[4], o[5], clear_grid_gradients=False)
    torch.cuda.synchronize()
    np.testing.assert_allclose(o[0].cpu().numpy(), r[0].cpu().numpy(), rtol=2e-6, atol=1e-8)
    assert (o[5].cpu().numpy() == r[5].cpu().numpy()).all()


def _synthetic_output(coords: np.ndarray) -> np.ndarray:
    """A smooth deterministic 'network output' per sample record (raw rgb, raw density)."""
    out = np.zeros((coords.shape[0], 16), np.float16)
    x, y, z = coords[:, 0], coords[:, 1], coords[:, 2]
    out[:, 0] = np.sin(7 * x) * 2
    out[:, 1] = np.cos(5 * y) * 2
    out[:, 2] = (z - 0.5) * 4
    out[:, 3] = np.sin(3 * x + 2 * y) * 4 + 1.5
    return out


def test_training_loss_vs_reference_kernel(ngp, reflib, small_scene, blob_bitfield):
    """compute_training_loss_and_compact_kernel vs ours on the same rays and network outputs:
    per-ray loss, compacted count and per-sample gradients (rays matched by index)."""
    import torch

    pix, cam, tr = _scene_tensors(small_scene)
    F, H, W = tr["pixels"].shape[:3]
    bits = T(blob_bitfield)
    n, limit, step = 4096, 1 << 20, 11
    (fx, fy), (cx, cy) = tr["focal"], tr["principal"]
    # ours: march, outputs, loss
    ns = torch.zeros((n, 2), dtype=torch.int32, device="cuda")
    rays = torch.zeros((n, 6), dtype=torch.float32, device="cuda")
    ridx = torch.zeros(n, dtype=torch.int32, device="cuda")
    coords = torch.zeros((limit, 7), dtype=torch.float32, device="cuda")
    totals = torch.zeros(ngp.march_scratch_words(n), dtype=torch.int32, device="cuda")
    rc = torch.zeros(1, dtype=torch.int32, device="cuda")
    sc = torch.zeros(1, dtype=torch.int32, device="cuda")
    ngp.march_training_rays(cam, F, W, H, fx, fy, cx, cy, step, n, limit, bits, coords, rays, ridx, ns, totals, rc, sc)
    torch.cuda.synchronize()
    total = int(sc.item())
    out = T(np.concatenate([_synthetic_output(coords[:total].cpu().numpy()), np.zeros((limit - total, 16), np.float16)]))
    ccoords = torch.zeros((1 << 18, 7), dtype=torch.float32, device="cuda")
    dloss = torch.zeros((1 << 18, 16), dtype=torch.float16, device="cuda")
    loss = torch.zeros(n, dtype=torch.float32, device="cuda")
    cc = torch.zeros(1, dtype=torch.int32, device="cuda")
    scratch = torch.zeros(ngp.loss_scratch_bytes(n), dtype=torch.uint8, device="cuda")
    ngp.training_loss_and_compact(n, step, rc, pix, F, W, H, out, cc, ridx, rays, ns, coords, ccoords, dloss, loss, scratch)
    # reference: its own march, same output function, its loss kernel
    r_rc = torch.zeros(1, dtype=torch.int32, device="cuda")
    r_sc = torch.zeros(1, dtype=torch.int32, device="cuda")
    r_idx = torch.zeros(n, dtype=torch.int32, device="cuda")
    r_rays = torch.zeros((n, 6), dtype=torch.float32, device="cuda")
    r_ns = torch.zeros((n, 2), dtype=torch.int32, device="cuda")
    r_coords = torch.zeros((limit, 7), dtype=torch.float32, device="cuda")
    reflib.call("ref_generate_training_samples", ctypes.c_uint32(n), ctypes.c_uint32(limit), ctypes.c_uint32(step), ctypes.c_uint32(F),
                ctypes.c_uint32(W), ctypes.c_uint32(H), ctypes.c_float(fx), ctypes.c_float(fy), ctypes.c_float(cx), ctypes.c_float(cy), P(cam),
                P(bits), P(r_rc), P(r_sc), P(r_idx), P(r_rays), P(r_ns), P(r_coords))
    r_out = T(np.concatenate([_synthetic_output(r_coords[:total].cpu().numpy()), np.zeros((limit - total, 16), np.float16)]))
    r_cc = torch.zeros(1, dtype=torch.int32, device="cuda")
    r_ccoords = torch.zeros_like(ccoords)
    r_dloss = torch.zeros_like(dloss)
    r_loss = torch.zeros(n, dtype=torch.float32, device="cuda")
    reflib.call("ref_training_loss", ctypes.c_uint32(n), ctypes.c_uint32(step), P(r_rc), P(pix), ctypes.c_uint32(F), ctypes.c_uint32(W),
                ctypes.c_uint32(H), P(r_out), P(r_cc), P(r_idx), P(r_rays), P(r_ns), P(r_coords), P(r_ccoords), P(r_dloss), P(r_loss))
    torch.cuda.synchronize()
    assert int(cc.item()) == int(r_cc.item())
    k = int(r_rc.item())
    ri = r_idx[:k].cpu().numpy()
    rns = r_ns[:k].cpu().numpy()
    ons = ns.cpu().numpy()
    assert (ons[ri, 0] == rns[:, 0]).all()  # compacted counts per ray
    ol = loss.cpu().numpy()
    rl = r_loss[:k].cpu().numpy()
    np.testing.assert_allclose(ol[ri], rl, rtol=1e-5, atol=1e-9)
    od = dloss.float().cpu().numpy()
    rd = r_dloss.float().cpu().numpy()
    oc = ccoords.cpu().numpy()
    rcc = r_ccoords.cpu().numpy()
    for j in range(k):
        c = rns[j, 0]
        a, b = rns[j, 1], ons[ri[j], 1]
        assert rcc[a: a + c].tobytes() == oc[b: b + c].tobytes()
        x, y = od[b: b + c, :4], rd[a: a + c, :4]
        assert (np.abs(x - y) <= 2e-3 * np.abs(y) + 1e-7).all(), j


def test_density_first_flow_matches_loss_and_compact(ngp, small_scene, blob_bitfield):
    """The trainer's density-first flow (density network on every sample, compaction, full network
    on the compacted rows, loss) against the one-pass entry point given the full network's
    outputs: counts, compacted records and encodings (after padding) bit-identical, including the
    ray that straddles the end of the 2^18 batch; losses and output gradients equal up to the
    association of the compositing sums (the one-pass kernel walks each ray in one warp, the
    compacted one splits long rays across warps and scans each chunk): 1e-5 relative on the
    loss, 2e-3 relative on the fp16 gradients, as against the reference kernel."""
    import torch

    pix, cam, tr = _scene_tensors(small_scene)
    F, H, W = tr["pixels"].shape[:3]
    bits = T(blob_bitfield)
    n, limit, step, batch = 12288, 1 << 21, 5, 1 << 18
    rows = ngp.compacted_rows()
    assert rows == batch + 1024
    (fx, fy), (cx, cy) = tr["focal"], tr["principal"]
    layout = ngp.grid_layout(16, 2, 19, 16, math.log2(128.0) / 15.0)
    _, table, _ = workloads.encode_inputs(1, layout.n_params, 16, 2, seed=4)
    table = (table.astype(np.float32) * 2e4).astype(np.float16)  # densities that end rays early
    table_t = T(table.view(np.int16))
    params = T(workloads.xavier_mlp_params(9).view(np.int16))
    ns = torch.zeros((n, 2), dtype=torch.int32, device="cuda")
    rays = torch.zeros((n, 6), dtype=torch.float32, device="cuda")
    ridx = torch.zeros(n, dtype=torch.int32, device="cuda")
    coords = torch.zeros((limit, 7), dtype=torch.float32, device="cuda")
    msc = torch.zeros(ngp.march_scratch_words(n), dtype=torch.int32, device="cuda")
    rc = torch.zeros(1, dtype=torch.int32, device="cuda")
    sc = torch.zeros(1, dtype=torch.int32, device="cuda")
    ngp.march_training_rays(cam, F, W, H, fx, fy, cx, cy, step, n, limit, bits, coords, rays, ridx, ns, msc, rc, sc)
    torch.cuda.synchronize()
    total = int(sc.item())
    m = (total + 127) // 128 * 128
    assert total > 2 * batch
    enc = torch.zeros((32, m), dtype=torch.float16, device="cuda")
    ngp.encode_grid_forward(layout, coords, table_t, enc, n=m, coord_stride=7, out_stride=m)
    scratch = torch.zeros(ngp.loss_scratch_bytes(n), dtype=torch.uint8, device="cuda")
    # one-pass flow
    out = torch.zeros((m, 16), dtype=torch.float16, device="cuda")
    ngp.mlp_forward(params, enc, coords, out, n=m, x_stride=m)
    ns_a = ns.clone()
    cc_a = torch.zeros(1, dtype=torch.int32, device="cuda")
    ccoords_a = torch.zeros((batch, 7), dtype=torch.float32, device="cuda")
    dloss_a = torch.zeros((batch, 16), dtype=torch.float16, device="cuda")
    loss_a = torch.zeros(n, dtype=torch.float32, device="cuda")
    ngp.training_loss_and_compact(n, step, rc, pix, F, W, H, out, cc_a, ridx, rays, ns_a, coords, ccoords_a, dloss_a, loss_a, scratch)
    ngp.pad_training_batch(cc_a, ccoords_a, dloss_a)
    cenc_a = torch.zeros((32, batch), dtype=torch.float16, device="cuda")
    ngp.encode_grid_forward(layout, ccoords_a, table_t, cenc_a, n=batch, coord_stride=7, out_stride=batch)
    # density-first flow
    dens = torch.zeros(m, dtype=torch.float16, device="cuda")
    ngp.density_forward(params, enc, dens, n=m, x_stride=m)
    ns_b = ns.clone()
    cc_b = torch.zeros(1, dtype=torch.int32, device="cuda")
    ccoords_b = torch.zeros((rows, 7), dtype=torch.float32, device="cuda")
    cenc_b = torch.zeros((32, rows), dtype=torch.float16, device="cuda")
    ngp.training_compact_by_density(n, rc, dens, coords, ns_b, ccoords_b, cc_b, scratch, enc=enc, enc_stride=m, compacted_enc=cenc_b)
    cout = torch.zeros((rows, 16), dtype=torch.float16, device="cuda")
    ngp.mlp_forward(params, cenc_b, ccoords_b, cout, n=rows, x_stride=rows)
    dloss_b = torch.zeros((batch, 16), dtype=torch.float16, device="cuda")
    loss_b = torch.zeros(n, dtype=torch.float32, device="cuda")
    ngp.training_loss_compacted(n, step, rc, pix, F, W, H, cout, ridx, rays, ns_b, ccoords_b, dloss_b, loss_b, scratch)
    ngp.pad_training_batch_enc(cc_b, ccoords_b, dloss_b, cenc_b, rows)
    torch.cuda.synchronize()
    assert int(cc_a.item()) == int(cc_b.item()) == batch
    assert (ns_a.cpu().numpy() == ns_b.cpu().numpy()).all()
    kept = ns_a.cpu().numpy()[:, 0]
    assert 0 < (kept > 0).sum() < n  # rays beyond the batch end were dropped
    assert ccoords_a.cpu().numpy().tobytes() == ccoords_b[:batch].cpu().numpy().tobytes()
    x, y = dloss_a.float().cpu().numpy(), dloss_b.float().cpu().numpy()
    assert (np.abs(x - y) <= 2e-3 * np.abs(y) + 1e-7).all()
    np.testing.assert_allclose(loss_a.cpu().numpy(), loss_b.cpu().numpy(), rtol=1e-5, atol=1e-9)
    assert cenc_a.cpu().numpy().view(np.uint16).tobytes() == cenc_b[:, :batch].cpu().numpy().view(np.uint16).tobytes()
    # some rays stopped early (transmittance), so the flow's keep decision was exercised
    steps = ns.cpu().numpy()[:, 0]
    assert (kept[kept > 0] < steps[kept > 0]).any()


def test_progressive_density_evaluation_matches_full(ngp, small_scene, blob_bitfield):
    """Densities evaluated only in front of each ray's stopping point (first 48 samples of every
    ray, then the rest of the rays still going) give the same kept counts, compacted records and
    encodings as evaluating every marched sample, bit for bit, including the ray straddling the
    2^18 end and rays that stop inside and after the first round."""
    import torch

    pix, cam, tr = _scene_tensors(small_scene)
    F, H, W = tr["pixels"].shape[:3]
    bits = T(blob_bitfield)
    n, limit, step, batch = 12288, 1 << 21, 6, 1 << 18
    rows_n = ngp.compacted_rows()
    (fx, fy), (cx, cy) = tr["focal"], tr["principal"]
    layout = ngp.grid_layout(16, 2, 19, 16, math.log2(128.0) / 15.0)
    _, table, _ = workloads.encode_inputs(1, layout.n_params, 16, 2, seed=4)
    table = (table.astype(np.float32) * 2e4).astype(np.float16)
    mlp = workloads.xavier_mlp_params(9)
    # raw density = positive weights . ReLU(hidden): rays stop after tens of samples, some inside
    # the first round and some after it
    mlp[2048:2048 + 64] = np.random.default_rng(3).uniform(0.2, 0.5, 64).astype(np.float16)
    params = T(np.concatenate([mlp, table]).view(np.int16))
    ns = torch.zeros((n, 2), dtype=torch.int32, device="cuda")
    rays = torch.zeros((n, 6), dtype=torch.float32, device="cuda")
    ridx = torch.zeros(n, dtype=torch.int32, device="cuda")
    coords = torch.zeros((limit, 7), dtype=torch.float32, device="cuda")
    msc = torch.zeros(ngp.march_scratch_words(n), dtype=torch.int32, device="cuda")
    rc = torch.zeros(1, dtype=torch.int32, device="cuda")
    sc = torch.zeros(1, dtype=torch.int32, device="cuda")
    ngp.march_training_rays(cam, F, W, H, fx, fy, cx, cy, step, n, limit, bits, coords, rays, ridx, ns, msc, rc, sc)
    torch.cuda.synchronize()
    total = int(sc.item())
    m = (total + 127) // 128 * 128
    scratch = torch.zeros(ngp.loss_scratch_bytes(n), dtype=torch.uint8, device="cuda")
    # every sample
    enc = torch.zeros((32, m), dtype=torch.float16, device="cuda")
    ngp.encode_grid_forward(layout, coords, params[10240:], enc, n=m, coord_stride=7, out_stride=m)
    dens = torch.zeros(m, dtype=torch.float16, device="cuda")
    ngp.density_forward(params[:10240], enc, dens, n=m, x_stride=m)
    ns_a, cc_a = ns.clone(), torch.zeros(1, dtype=torch.int32, device="cuda")
    cco_a = torch.zeros((rows_n, 7), dtype=torch.float32, device="cuda")
    cen_a = torch.zeros((32, rows_n), dtype=torch.float16, device="cuda")
    ngp.training_compact_by_density(n, rc, dens, coords, ns_a, cco_a, cc_a, scratch, enc=enc, enc_stride=m, compacted_enc=cen_a)
    kept_a = scratch[4 * n: 8 * n].view(torch.int32).clone()
    # progressive
    enc_b = torch.zeros((32, m), dtype=torch.float16, device="cuda")
    dens_b = torch.zeros(m, dtype=torch.float16, device="cuda")
    rows = torch.zeros(m, dtype=torch.int32, device="cuda")
    ns_b, cc_b = ns.clone(), torch.zeros(1, dtype=torch.int32, device="cuda")
    cco_b = torch.zeros((rows_n, 7), dtype=torch.float32, device="cuda")
    cen_b = torch.zeros((32, rows_n), dtype=torch.float16, device="cuda")
    ngp.training_compact_progressive(n, rc, layout, params, coords, m, ns_b, enc_b, dens_b, rows, cco_b, cen_b, cc_b, scratch)
    kept_b = scratch[4 * n: 8 * n].view(torch.int32).clone()
    torch.cuda.synchronize()
    assert int(cc_a.item()) == int(cc_b.item()) == batch
    assert (kept_a == kept_b).all()
    assert (ns_a == ns_b).all()
    assert cco_a.cpu().numpy().tobytes() == cco_b.cpu().numpy().tobytes()
    assert cen_a.cpu().numpy().view(np.uint16).tobytes() == cen_b.cpu().numpy().view(np.uint16).tobytes()
    steps = ns.cpu().numpy()[:, 0]
    kept = kept_a.cpu().numpy()
    stop0 = int(((kept < 48) & (kept < steps)).sum())
    stop1 = int(((kept > 48) & (kept < steps)).sum())
    assert stop0 > 0 and stop1 > 0, (stop0, stop1, np.percentile(kept[steps > 0], [10, 50, 90]))  # stops in both rounds
    evaluated = int((dens_b != 0).sum().item())
    assert evaluated < total  # densities only in front of the stopping points


def test_progressive_evaluation_renders_identically(ngp, small_scene, blob_bitfield):
    """Rendering with network outputs only in front of each ray's stopping point gives the same
    image, bit for bit, as evaluating every marched sample (the compositing stops where the
    progressive evaluation stops)."""
    import torch

    _, cam, tr = _scene_tensors(small_scene)
    F, H, W = tr["pixels"].shape[:3]
    (fx, fy), (cx, cy) = tr["focal"], tr["principal"]
    layout = ngp.grid_layout(16, 2, 19, 16, math.log2(128.0) / 15.0)
    _, table, _ = workloads.encode_inputs(1, layout.n_params, 16, 2, seed=4)
    table = (table.astype(np.float32) * 2e4).astype(np.float16)
    mlp = workloads.xavier_mlp_params(9)
    mlp[2048:2048 + 64] = np.random.default_rng(3).uniform(0.2, 0.5, 64).astype(np.float16)
    params = T(np.concatenate([mlp, table]).view(np.int16))
    n = W * H
    rays = torch.zeros((n, 6), dtype=torch.float32, device="cuda")
    ngp.make_eval_rays(cam, 0, W, H, fx, fy, cx, cy, 0, n, rays)
    limit = 1 << 21
    coords = torch.zeros((limit, 7), dtype=torch.float32, device="cuda")
    ns = torch.zeros((n, 2), dtype=torch.int32, device="cuda")
    msc = torch.zeros(ngp.march_scratch_words(n), dtype=torch.int32, device="cuda")
    sc = torch.zeros(1, dtype=torch.int32, device="cuda")
    ngp.march_rays(rays, T(blob_bitfield), coords, ns, msc, sc, sample_limit=limit)
    torch.cuda.synchronize()
    total = int(sc.item())
    m = (total + 127) // 128 * 128
    enc = torch.zeros((32, m), dtype=torch.float16, device="cuda")
    full = torch.zeros((m, 16), dtype=torch.float16, device="cuda")
    ngp.encode_grid_forward(layout, coords, params[10240:], enc, n=m, coord_stride=7, out_stride=m)
    ngp.mlp_forward(params[:10240], enc, coords, full, n=m, x_stride=m)
    prog = torch.zeros((m, 16), dtype=torch.float16, device="cuda")
    enc2 = torch.zeros((32, m), dtype=torch.float16, device="cuda")
    rows = torch.zeros(m, dtype=torch.int32, device="cuda")
    scratch = torch.zeros(ngp.loss_scratch_bytes(n), dtype=torch.uint8, device="cuda")
    ngp.eval_network_progressive(n, layout, params, coords, m, ns, enc2, prog, rows, scratch)
    img_a = torch.zeros((n, 3), dtype=torch.float32, device="cuda")
    img_b = torch.zeros((n, 3), dtype=torch.float32, device="cuda")
    ngp.eval_composite(n, 0, 0, W, H, None, ns, coords, full, rendered=img_a)
    ngp.eval_composite(n, 0, 0, W, H, None, ns, coords, prog, rendered=img_b)
    torch.cuda.synchronize()
    assert img_a.cpu().numpy().tobytes() == img_b.cpu().numpy().tobytes()
    evaluated = int((prog[:total, 3] != 0).sum().item())
    assert 0 < evaluated < total


def test_selected_batch_matches_compacted_batch(ngp, small_scene, blob_bitfield):
    """The trainer's selection flow (the batch as a list of the kept samples' rows, network,
    loss and backward reading the samples in place) against the copying flow: same counts, the
    listed rows are the copied records and encodings, and the loss, output gradients, MLP weight
    gradients and input gradients are bit-identical; the grid gradient (fp32 atomics, summation
    order free) agrees within 1e-5 relative."""
    import torch

    pix, cam, tr = _scene_tensors(small_scene)
    F, H, W = tr["pixels"].shape[:3]
    bits = T(blob_bitfield)
    n, limit, step, batch = 12288, 1 << 21, 8, 1 << 18
    rows_n = ngp.compacted_rows()
    (fx, fy), (cx, cy) = tr["focal"], tr["principal"]
    layout = ngp.grid_layout(16, 2, 19, 16, math.log2(128.0) / 15.0)
    _, table, _ = workloads.encode_inputs(1, layout.n_params, 16, 2, seed=4)
    table = (table.astype(np.float32) * 2e4).astype(np.float16)
    mlp = workloads.xavier_mlp_params(9)
    mlp[2048:2048 + 64] = np.random.default_rng(3).uniform(0.2, 0.5, 64).astype(np.float16)
    params = T(np.concatenate([mlp, table]).view(np.int16))
    ns = torch.zeros((n, 2), dtype=torch.int32, device="cuda")
    rays = torch.zeros((n, 6), dtype=torch.float32, device="cuda")
    ridx = torch.zeros(n, dtype=torch.int32, device="cuda")
    coords = torch.zeros((limit, 7), dtype=torch.float32, device="cuda")
    msc = torch.zeros(ngp.march_scratch_words(n), dtype=torch.int32, device="cuda")
    rc = torch.zeros(1, dtype=torch.int32, device="cuda")
    sc = torch.zeros(1, dtype=torch.int32, device="cuda")
    ngp.march_training_rays(cam, F, W, H, fx, fy, cx, cy, step, n, limit, bits, coords, rays, ridx, ns, msc, rc, sc)
    torch.cuda.synchronize()
    m = (int(sc.item()) + 127) // 128 * 128

    def fresh(dtype, *shape):
        return torch.zeros(shape, dtype=dtype, device="cuda")

    # copying flow
    sa = fresh(torch.uint8, ngp.loss_scratch_bytes(n))
    ns_a, cc_a = ns.clone(), fresh(torch.int32, 1)
    enc_a, dens_a, rows_a = fresh(torch.float16, 32, m), fresh(torch.float16, m), fresh(torch.int32, m)
    cco, cen = fresh(torch.float32, rows_n, 7), fresh(torch.float16, 32, rows_n)
    ngp.training_compact_progressive(n, rc, layout, params, coords, m, ns_a, enc_a, dens_a, rows_a, cco, cen, cc_a, sa)
    out_a = fresh(torch.float16, rows_n, 16)
    ngp.mlp_forward(params[:10240], cen, cco, out_a, n=rows_n, x_stride=rows_n)
    dl_a, loss_a = fresh(torch.float16, batch, 16), fresh(torch.float32, n)
    ngp.training_loss_compacted(n, step, rc, pix, F, W, H, out_a, ridx, rays, ns_a, cco, dl_a, loss_a, sa)
    ngp.pad_training_batch_enc(cc_a, cco, dl_a, cen, rows_n)
    dx_a, dw_a = fresh(torch.float16, 32, batch), fresh(torch.float32, 10240)
    ngp.mlp_backward(params[:10240], cen, cco, dl_a, dx=dx_a, dw_f32=dw_a, n=batch, x_stride=rows_n)
    g_a = fresh(torch.float32, layout.n_params)
    ngp.encode_grid_backward(layout, cco, dx_a, g_a, n=batch, coord_stride=7)
    # selection flow
    sb = fresh(torch.uint8, ngp.loss_scratch_bytes(n))
    ns_b, cc_b, nsel = ns.clone(), fresh(torch.int32, 1), fresh(torch.int32, 1)
    enc_b, dens_b, rows_b, brows = fresh(torch.float16, 32, m), fresh(torch.float16, m), fresh(torch.int32, m), fresh(torch.int32, rows_n)
    ngp.training_select_progressive(n, rc, layout, params, coords, m, ns_b, enc_b, dens_b, rows_b, brows, nsel, cc_b, sb)
    out_b = fresh(torch.float16, m, 16)
    ngp.mlp_forward_rows(rows_n, brows, nsel, params[:10240], enc_b, m, coords, out_b)
    dl_b, loss_b = fresh(torch.float16, batch, 16), fresh(torch.float32, n)
    ngp.training_loss_selected(n, step, rc, pix, F, W, H, out_b, ridx, rays, ns_b, coords, dl_b, loss_b, sb)
    ngp.pad_training_rows(cc_b, brows, dl_b)
    dx_b, dw_b = fresh(torch.float16, 32, batch), fresh(torch.float32, 10240)
    ngp.mlp_backward_rows(batch, brows, params[:10240], enc_b, m, coords, dl_b, dx_b, batch, dw_b)
    g_b = fresh(torch.float32, layout.n_params)
    ngp.encode_grid_backward_rows(layout, batch, brows, coords, dx_b, g_b)
    torch.cuda.synchronize()
    assert int(cc_a.item()) == int(cc_b.item()) == batch
    assert (ns_a == ns_b).all()
    rb = brows[:batch].long()
    assert cco[:batch].cpu().numpy().tobytes() == coords[rb].cpu().numpy().tobytes()
    assert cen[:, :batch].cpu().numpy().view(np.uint16).tobytes() == enc_b[:, rb].cpu().numpy().view(np.uint16).tobytes()
    assert loss_a.cpu().numpy().tobytes() == loss_b.cpu().numpy().tobytes()
    assert dl_a.cpu().numpy().view(np.uint16).tobytes() == dl_b.cpu().numpy().view(np.uint16).tobytes()
    assert dw_a.cpu().numpy().tobytes() == dw_b.cpu().numpy().tobytes()
    assert dx_a.cpu().numpy().view(np.uint16).tobytes() == dx_b.cpu().numpy().view(np.uint16).tobytes()
    ga, gb = g_a.cpu().numpy(), g_b.cpu().numpy()
    assert np.abs(ga - gb).max() <= 1e-5 * np.abs(ga).max()


@pytest.mark.parametrize("sets", [(1 << 21, 0), (1 << 19, 1 << 19), (1 << 16, 3000)], ids=["warm-up", "steady", "ragged"])
def test_grid_samples_cell_order_is_a_permutation_of_the_reference(ngp, reflib, sets):
    """The cell-ordered samples are the reference kernel's samples (same records and cell indices,
    bit for bit) in another order; warps hold consecutive first cells."""
    import torch

    nu, nn = sets
    vals0 = workloads.blob_grid_values(workloads.gaussian_blob_density())
    vals0[::97] = -1.0  # untrained cells: the uniform samples there retry elsewhere
    values = T(vals0)
    n = nu + nn
    coords = torch.zeros((n, 7), dtype=torch.float32, device="cuda")
    idx = torch.zeros(n, dtype=torch.int32, device="cuda")
    counter = torch.zeros(1, dtype=torch.int32, device="cuda")
    ngp.density_grid_samples_cell_order(nu, nn, 7, values, coords, idx, counter)
    rcoords = torch.zeros_like(coords)
    ridx = torch.zeros_like(idx)
    reflib.call("ref_grid_samples", ctypes.c_uint32(nu), ctypes.c_uint32(nn), ctypes.c_uint32(7), P(values), P(rcoords), P(ridx))
    torch.cuda.synchronize()
    if nn:
        assert int(counter.item()) == n

    def rows(c, i):
        return np.concatenate([c.cpu().numpy().view(np.uint32), i.cpu().numpy().view(np.uint32)[:, None]], axis=1)

    a, b = rows(coords, idx), rows(rcoords, ridx)
    a, b = a[np.lexsort(a.T[::-1])], b[np.lexsort(b.T[::-1])]
    assert np.array_equal(a, b)
    if nu == 1 << 21 and nn == 0:
        # slot g holds the sample whose first cell is g: cells ascend wherever no retry happened
        cells = idx.cpu().numpy().view(np.uint32)
        assert (cells == np.arange(n, dtype=np.uint32)).mean() > 0.95


@pytest.mark.parametrize("layout_args", [(16, 2, 19, 16, math.log2(2048.0 / 16.0) / 15.0), (8, 4, 19, 16, 1.0)], ids=["16x2", "8x4"])
@pytest.mark.parametrize("ema_step", [0, 7])
def test_grid_encode_samples_equals_samples_then_encode(ngp, layout_args, ema_step):
    """ngp_density_grid_encode_samples (warm-up samples made inside the encoding kernel) against
    the cell-ordered samples followed by the encoding of their records: encodings and cell
    indices bit for bit, untrained cells (retries) included."""
    import torch

    n = 1 << 21
    layout = ngp.grid_layout(*layout_args)
    _, table, _ = workloads.encode_inputs(1, layout.n_params, layout_args[0], layout_args[1], seed=11)
    table_t = T(table.view(np.int16))
    vals0 = workloads.blob_grid_values(workloads.gaussian_blob_density())
    vals0[::97] = -1.0
    values = T(vals0)
    coords = torch.zeros((n, 7), dtype=torch.float32, device="cuda")
    idx_a = torch.zeros(n, dtype=torch.int32, device="cuda")
    ngp.density_grid_samples_cell_order(n, 0, ema_step, values, coords, idx_a)
    F = layout_args[0] * layout_args[1]
    enc_a = torch.zeros((F, n), dtype=torch.float16, device="cuda")
    ngp.encode_grid_forward(layout, coords, table_t, enc_a, n=n, coord_stride=7, out_stride=n)
    enc_b = torch.zeros_like(enc_a)
    idx_b = torch.zeros_like(idx_a)
    ngp.density_grid_encode_samples(layout, ema_step, values, table_t, enc_b, idx_b)
    torch.cuda.synchronize()
    assert torch.equal(idx_a, idx_b)
    assert enc_a.cpu().numpy().view(np.uint16).tobytes() == enc_b.cpu().numpy().view(np.uint16).tobytes()


def test_density_forward_splat_equals_forward_then_splat(ngp):
    """The density network with the grid splat in its epilogue against ngp_density_forward followed
    by ngp_density_grid_splat: the splatted grid bit for bit (cells hit by several samples
    included)."""
    import torch

    n = 1 << 20
    x_h, _, _ = workloads.mlp_inputs(n, seed=21)
    params = T(workloads.xavier_mlp_params(3).view(np.int16))
    x = T(x_h)
    rng = np.random.default_rng(5)
    cells = rng.integers(0, 128 ** 3, n).astype(np.int32)  # random cells: some repeat
    idx = T(cells)
    dens = torch.zeros(n, dtype=torch.float16, device="cuda")
    ngp.density_forward(params, x, dens, n=n)
    a = torch.zeros(128 ** 3, dtype=torch.float32, device="cuda")
    ngp.density_grid_splat(n, idx, dens, a)
    b = torch.zeros_like(a)
    ngp.density_forward_splat(params, x, idx, b, n=n)
    torch.cuda.synchronize()
    assert (a > 0).sum().item() > 0.3 * n
    assert a.cpu().numpy().tobytes() == b.cpu().numpy().tobytes()


def test_selection_does_not_depend_on_the_first_window(ngp, small_scene, blob_bitfield):
    """ngp_training_select_progressive_window: one round (window = all samples), the default 48
    and a narrow 5-sample window select the same batch (rows, counts, compacted counter,
    numsteps); still_active counts the rays that outlive the first window."""
    import torch

    pix, cam, tr = _scene_tensors(small_scene)
    F, H, W = tr["pixels"].shape[:3]
    bits = T(blob_bitfield)
    n, limit, step = 12288, 1 << 21, 8
    rows_n = ngp.compacted_rows()
    (fx, fy), (cx, cy) = tr["focal"], tr["principal"]
    layout = ngp.grid_layout(16, 2, 19, 16, math.log2(128.0) / 15.0)
    _, table, _ = workloads.encode_inputs(1, layout.n_params, 16, 2, seed=4)
    table = (table.astype(np.float32) * 2e4).astype(np.float16)
    params = T(np.concatenate([workloads.xavier_mlp_params(9), table]).view(np.int16))
    ns = torch.zeros((n, 2), dtype=torch.int32, device="cuda")
    rays = torch.zeros((n, 6), dtype=torch.float32, device="cuda")
    ridx = torch.zeros(n, dtype=torch.int32, device="cuda")
    coords = torch.zeros((limit, 7), dtype=torch.float32, device="cuda")
    msc = torch.zeros(ngp.march_scratch_words(n), dtype=torch.int32, device="cuda")
    rc = torch.zeros(1, dtype=torch.int32, device="cuda")
    sc = torch.zeros(1, dtype=torch.int32, device="cuda")
    ngp.march_training_rays(cam, F, W, H, fx, fy, cx, cy, step, n, limit, bits, coords, rays, ridx, ns, msc, rc, sc)
    torch.cuda.synchronize()
    m = (int(sc.item()) + 127) // 128 * 128
    out = {}
    for window in (0xFFFFFFFF, 48, 5):
        z = lambda dtype, *shape: torch.zeros(shape, dtype=dtype, device="cuda")  # noqa: E731
        ns_w, cc, nsel, active = ns.clone(), z(torch.int32, 1), z(torch.int32, 1), z(torch.int32, 1)
        active.fill_(12345)
        enc, dens, rows, brows = z(torch.float16, 32, m), z(torch.float16, m), z(torch.int32, m), z(torch.int32, rows_n)
        scratch = z(torch.uint8, ngp.loss_scratch_bytes(n))
        ngp.training_select_progressive_window(n, rc, layout, params, coords, m, ns_w, enc, dens, rows, brows, nsel, cc, scratch, window, active)
        torch.cuda.synchronize()
        out[window] = (ns_w.cpu().numpy(), int(cc.item()), int(nsel.item()), brows[: int(nsel.item())].cpu().numpy(), int(active.item()))
    a = out[0xFFFFFFFF]
    for window in (48, 5):
        b = out[window]
        assert (a[0] == b[0]).all() and a[1] == b[1] and a[2] == b[2] and np.array_equal(a[3], b[3])
    assert a[4] == 0  # one round: nothing left for a second
    rays_n = int(rc.item())
    assert 0 < out[5][4] <= rays_n and out[48][4] <= out[5][4]
