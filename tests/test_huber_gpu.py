"""Huber loss variant of the training loss (ngp_training_loss_selected_kind, loss_kind 1): the
loss of the original instant-ngp NeRF, delta 0.1, divided by 5 so that it equals the L2 loss for
residuals |d| <= 0.1 (the reference's L2 site: ngp.train.cu:817-820).  Reported separately from
the L2 parity runs.

Checked against a numpy restatement of the compositing backward (K11's per-sample gradients,
ngp.train.cu:804-859, with the Huber derivative in place of 2 d) on a scene whose every pixel has
one opaque colour, so the target of every ray is known on the host; rays whose samples were all
kept (their colour includes the random background) are left out.  Tolerances: loss 1e-4
relative, fp16 gradients 3e-3 relative + 1e-6.  L2 through the same entry point equals the
reference-mirroring ngp_training_loss_selected bit for bit."""
from __future__ import annotations

import math

import numpy as np
import pytest

import workloads

pytestmark = pytest.mark.gpu


def T(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _srgb_to_linear(v):
    return np.where(v <= 0.04045, v / 12.92, ((v + 0.055) / 1.055) ** 2.4)


def _linear_to_srgb(v):
    return np.where(v < 0.0031308, 12.92 * v, 1.055 * v ** 0.41666 - 0.055)


def _sig(x):
    return 1.0 / (1.0 + np.exp(-x))


def _huber_grad(d):
    return np.where(np.abs(d) <= 0.1, 2.0 * d, 0.2 * np.sign(d))


def _huber(d):
    a = np.abs(d)
    return np.where(a <= 0.1, d * d, 0.2 * a - 0.01)


def test_huber_loss_matches_restatement(ngp):
    import torch

    scene = workloads.procedural_dataset(n_train=6, n_test=1, width=96, height=80, seed=5)
    tr = scene["train"]
    F, H, W = tr["pixels"].shape[:3]
    colour = np.array([200, 120, 40], np.uint8)
    px = np.zeros((F, H, W, 4), np.uint8)
    px[..., :3] = colour
    px[..., 3] = 255
    pix, cam = T(px), T(tr["camera"])
    n, limit, step, batch = 4096, 1 << 21, 5, 1 << 18
    (fx, fy), (cx, cy) = tr["focal"], tr["principal"]
    bits = torch.full((128 ** 3 // 8,), 0xFF, dtype=torch.uint8, device="cuda")
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
    rows_n = ngp.compacted_rows()

    def fresh(dtype, *shape):
        return torch.zeros(shape, dtype=dtype, device="cuda")

    sb = fresh(torch.uint8, ngp.loss_scratch_bytes(n))
    ns_sel, cc, nsel = ns.clone(), fresh(torch.int32, 1), fresh(torch.int32, 1)
    enc, dens, rows, brows = fresh(torch.float16, 32, m), fresh(torch.float16, m), fresh(torch.int32, m), fresh(torch.int32, rows_n)
    ngp.training_select_progressive(n, rc, layout, params, coords, m, ns_sel, enc, dens, rows, brows, nsel, cc, sb)
    out = fresh(torch.float16, m, 16)
    ngp.mlp_forward_rows(rows_n, brows, nsel, params[:10240], enc, m, coords, out)
    res = {}
    for kind in (0, 1):
        nsk, dl, loss = ns_sel.clone(), fresh(torch.float16, batch, 16), fresh(torch.float32, n)
        ngp.training_loss_selected_kind(n, step, rc, pix, F, W, H, out, ridx, rays, nsk, coords, dl, loss, sb, kind)
        res[kind] = (nsk.cpu().numpy(), dl.float().cpu().numpy(), loss.cpu().numpy())
    nsl, dll, lossl = ns_sel.clone(), fresh(torch.float16, batch, 16), fresh(torch.float32, n)
    ngp.training_loss_selected(n, step, rc, pix, F, W, H, out, ridx, rays, nsl, coords, dll, lossl, sb)
    torch.cuda.synchronize()
    assert np.array_equal(dll.float().cpu().numpy(), res[0][1]) and np.array_equal(lossl.cpu().numpy(), res[0][2])

    march = ns.cpu().numpy()
    kept_sel = ns_sel.cpu().numpy()[:, 0]
    o = out.float().cpu().numpy().astype(np.float64)
    c = coords.cpu().numpy().astype(np.float64)
    target = _linear_to_srgb(_srgb_to_linear(colour.astype(np.float64) / 255.0))
    scale = 128.0 / n
    nsh, dlh, lossh = res[1]
    checked = 0
    big = 0
    for i in range(int(rc.item())):
        cnt, base = int(march[i, 0]), int(march[i, 1])
        k = int(kept_sel[i])
        cn, cbase = int(nsh[i, 0]), int(nsh[i, 1])
        if k == 0 or k >= cnt or cn == 0:
            continue  # all samples kept: the colour includes the random background
        rgb_raw, md, dt = o[base:base + k, :3], o[base:base + k, 3], c[base:base + k, 3]
        alpha = 1.0 - np.exp(-np.exp(md) * dt)
        Tb = np.concatenate([[1.0], np.cumprod(1.0 - alpha)[:-1]])
        w = alpha * Tb
        col = _sig(rgb_raw)
        rgb = (w[:, None] * col).sum(0)
        d = rgb - target
        big += int((np.abs(d) > 0.12).any())
        assert abs(lossh[i] - _huber(d).sum() / (3 * n)) <= 1e-4 * _huber(d).sum() / (3 * n) + 1e-9
        g = _huber_grad(d)
        prefix = np.cumsum(w[:, None] * col, axis=0)
        Ta = Tb * (1.0 - alpha)
        want_rgb = scale * w[:, None] * g[None, :] * col * (1.0 - col)
        want_d = scale * np.exp(np.clip(md, -15, 15)) * dt * ((Ta[:, None] * col - (rgb[None, :] - prefix)) * g[None, :]).sum(1)
        got = dlh[cbase:cbase + cn]
        np.testing.assert_allclose(got[:, :3], want_rgb[:cn], rtol=3e-3, atol=1e-6)
        np.testing.assert_allclose(got[:, 3], want_d[:cn], rtol=3e-3, atol=2e-5)
        checked += 1
    assert checked > 100 and big > 10
