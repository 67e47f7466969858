"""Hash-grid encoding parity: CUDA library vs CPU oracle vs the reference's own kernels.

Tolerances (north_star: encoding outputs and gradients within 1e-3 relative, fp16):
* forward, library vs oracle: bit-exact (same fp32 fmaf chain, one rounding to fp16);
* forward, reference kernel vs oracle in reference mode: bit-exact (fp16 __hfma chain);
* forward, library vs reference kernel: |a - b| <= 1e-3 * |b| + 16 fp16 subnormal ulps (the reference
  accumulates in fp16, the library in fp32);
* backward, library (fp32 atomics) vs oracle (fp64 sums): |a - b| <= 1e-3 * |b| + 1e-6 * max|b|.
"""
from __future__ import annotations

import math

import numpy as np
import pytest

import workloads

pytestmark = pytest.mark.gpu

CFG0 = (16, 2, 19, 16, math.log2(128.0) / 15.0)
REF = (8, 4, 19, 16, 1.0)


def _torch():
    import torch

    return torch


def run_forward(ngp, layout, coords, table, F):
    torch = _torch()
    n = coords.shape[0]
    c = torch.from_numpy(coords).cuda()
    t = torch.from_numpy(table.view(np.int16)).cuda()
    out = torch.zeros((layout.n_levels * F, max(n, 1)), dtype=torch.float16, device="cuda")
    ngp.encode_grid_forward(layout, c, t, out, n=n, coord_stride=coords.shape[1], out_stride=max(n, 1))
    torch.cuda.synchronize()
    return out.cpu().numpy()[:, :n]


def run_backward(ngp, layout, coords, dy, F):
    torch = _torch()
    c = torch.from_numpy(coords).cuda()
    g = torch.from_numpy(dy).cuda()
    grad = torch.zeros(layout.n_params, dtype=torch.float32, device="cuda")
    ngp.encode_grid_backward(layout, c, g, grad, n=coords.shape[0], coord_stride=coords.shape[1], dy_stride=dy.shape[1])
    torch.cuda.synchronize()
    return grad.cpu().numpy()


@pytest.mark.parametrize("cfg", [CFG0, REF], ids=["config0", "reference"])
@pytest.mark.parametrize("n", [1, 7, 255, 513, 4096])
@pytest.mark.parametrize("stride", [3, 7])
def test_forward_bit_exact_vs_oracle(ngp, oracle, cfg, n, stride):
    L, F = cfg[0], cfg[1]
    layout = ngp.grid_layout(*cfg)
    coords, table, _ = workloads.encode_inputs(n, layout.n_params, L, F, seed=n + stride, coord_stride=stride)
    got = run_forward(ngp, layout, coords, table, F)
    want = oracle.encode_forward(oracle.grid_layout(*cfg), coords, table, F, mode=0)
    assert got.view(np.uint16).tobytes() == want.view(np.uint16).tobytes()


def test_forward_edges_bit_exact(ngp, oracle):
    """Points on the cube's faces and corners, where the +1 corner reaches x == resolution."""
    layout = ngp.grid_layout(*CFG0)
    vals = np.array([0.0, 1.0, 0.5, 1.0 - 2**-24, 2**-24, 0.999], np.float32)
    coords = np.array(np.meshgrid(vals, vals, vals, indexing="ij")).reshape(3, -1).T.copy()
    _, table, _ = workloads.encode_inputs(1, layout.n_params, 16, 2, seed=5)
    got = run_forward(ngp, layout, coords, table, 2)
    want = oracle.encode_forward(oracle.grid_layout(*CFG0), coords, table, 2, mode=0)
    assert got.view(np.uint16).tobytes() == want.view(np.uint16).tobytes()


def test_forward_full_size_sampled(ngp, oracle):
    """2^18 points (config 0): every 97th point checked bit-exactly against the oracle."""
    layout = ngp.grid_layout(*CFG0)
    n = 1 << 18
    coords, table, _ = workloads.encode_inputs(n, layout.n_params, 16, 2, seed=42)
    got = run_forward(ngp, layout, coords, table, 2)
    idx = np.arange(0, n, 97)
    want = oracle.encode_forward(oracle.grid_layout(*CFG0), coords[idx], table, 2, mode=0)
    assert got[:, idx].view(np.uint16).tobytes() == want.view(np.uint16).tobytes()


@pytest.mark.parametrize("cfg", [CFG0, REF], ids=["config0", "reference"])
@pytest.mark.parametrize("n", [1, 100, 4096])
def test_backward_vs_oracle(ngp, oracle, cfg, n):
    L, F = cfg[0], cfg[1]
    layout = ngp.grid_layout(*cfg)
    coords, _, dy = workloads.encode_inputs(n, layout.n_params, L, F, seed=7 * n + 1)
    got = run_backward(ngp, layout, coords, dy, F)
    want = oracle.encode_backward(oracle.grid_layout(*cfg), coords, dy, F)
    tol = 1e-3 * np.abs(want) + 1e-6 * np.abs(want).max()
    assert (np.abs(got - want) <= tol).all()
    assert ((got != 0) == (want != 0)).mean() > 0.999


@pytest.mark.parametrize("n", [37, 4000])
def test_backward_ray_ordered_points_vs_oracle(ngp, oracle, n):
    """Points along rays at the marching step (as training batches are laid out): neighbouring
    lanes share cells on the coarse levels, whose updates are summed inside the warp first."""
    layout = ngp.grid_layout(*CFG0)
    rng = np.random.default_rng(n)
    n_rays = max(1, n // 40)
    o = rng.uniform(0.2, 0.8, (n_rays, 3))
    d = rng.normal(size=(n_rays, 3))
    d /= np.linalg.norm(d, axis=1, keepdims=True)
    t = np.arange(40) * (math.sqrt(3.0) / 1024.0)
    pts = np.clip(o[:, None, :] + t[None, :, None] * d[:, None, :], 0.0, 1.0).reshape(-1, 3)[:n]
    coords = np.ascontiguousarray(pts, np.float32)
    dy = rng.normal(0, 1, (32, n)).astype(np.float16)
    got = run_backward(ngp, layout, coords, dy, 2)
    want = oracle.encode_backward(oracle.grid_layout(*CFG0), coords, dy, 2)
    tol = 1e-3 * np.abs(want) + 1e-6 * np.abs(want).max()
    assert (np.abs(got - want) <= tol).all()


def test_backward_full_size_level_sums(ngp):
    """2^18 points: the corner weights sum to one, so each level/feature's gradient sums to sum(dy)."""
    layout = ngp.grid_layout(*CFG0)
    n = 1 << 18
    coords, _, dy = workloads.encode_inputs(n, layout.n_params, 16, 2, seed=3)
    grad = run_backward(ngp, layout, coords, dy, 2).astype(np.float64)
    offs = layout.level_offsets()
    for l in range(16):
        lvl = grad[offs[l] * 2: offs[l + 1] * 2].reshape(-1, 2)
        want = dy[2 * l: 2 * l + 2].astype(np.float64).sum(axis=1)
        np.testing.assert_allclose(lvl.sum(axis=0), want, rtol=1e-4, atol=0.5)


def test_reference_kernel_pins_oracle_forward(ngp, oracle, reflib):
    """The reference's encode_grid_forward_kernel equals the oracle's reference mode bit for bit."""
    torch = _torch()
    layout = ngp.grid_layout(*REF)
    n = 4096
    coords, table, _ = workloads.encode_inputs(n, layout.n_params, 8, 4, seed=11, coord_stride=7)
    out = torch.zeros((32, n), dtype=torch.float16, device="cuda")
    c = torch.from_numpy(coords).cuda()
    t = torch.from_numpy(table.view(np.int16)).cuda()
    import ctypes

    reflib.call("ref_encode_forward", ctypes.c_uint32(n), ctypes.c_void_p(c.data_ptr()), ctypes.c_void_p(t.data_ptr()),
                ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(0))
    torch.cuda.synchronize()
    ref_out = out.cpu().numpy()
    want = oracle.encode_forward(oracle.grid_layout(*REF), coords, table, 4, mode=1)
    assert ref_out.view(np.uint16).tobytes() == want.view(np.uint16).tobytes()
    # and the library (fp32 accumulation) agrees with the reference within the stated tolerance
    ours = run_forward(ngp, layout, coords, table, 4).astype(np.float32)
    r = ref_out.astype(np.float32)
    assert (np.abs(ours - r) <= 1e-3 * np.abs(r) + 16 * 2.0**-24).all()


def test_reference_kernel_backward_close(ngp, oracle, reflib):
    torch = _torch()
    import ctypes

    layout = ngp.grid_layout(*REF)
    n = 2048
    coords, _, dy = workloads.encode_inputs(n, layout.n_params, 8, 4, seed=13, coord_stride=7)
    c = torch.from_numpy(coords).cuda()
    g = torch.from_numpy(dy).cuda()
    grad16 = torch.zeros(layout.n_params, dtype=torch.float16, device="cuda")
    reflib.call("ref_encode_backward", ctypes.c_uint32(n), ctypes.c_void_p(c.data_ptr()), ctypes.c_void_p(g.data_ptr()),
                ctypes.c_void_p(grad16.data_ptr()), ctypes.c_void_p(0))
    torch.cuda.synchronize()
    ref_grad = grad16.float().cpu().numpy()
    want = oracle.encode_backward(oracle.grid_layout(*REF), coords, dy, 4)
    ours = run_backward(ngp, layout, coords, dy, 4)
    # the reference sums in fp16 (weight and product rounded to fp16): a few fp16 ulps of the sum
    scale = np.abs(want).max()
    assert np.abs(ref_grad - want).max() <= 4e-3 * scale
    assert np.abs(ours - want).max() <= 1e-5 * scale


def test_invalid_arguments(ngp):
    torch = _torch()
    layout = ngp.grid_layout(*CFG0)
    c = torch.zeros((4, 3), device="cuda")
    assert ngp.lib().ngp_encode_grid_forward(None, 4, None, 3, None, None, 4, None) == 1
    assert b"null" in ngp.lib().ngp_last_error()
    with pytest.raises(RuntimeError, match="stride"):
        out = torch.zeros((32, 4), dtype=torch.float16, device="cuda")
        ngp.encode_grid_forward(layout, c, torch.zeros(layout.n_params, dtype=torch.float16, device="cuda"), out, coord_stride=2)
    # n == 0 is a no-op
    ngp.encode_grid_forward(layout, c, torch.zeros(1, dtype=torch.float16, device="cuda"), torch.zeros((32, 1), dtype=torch.float16, device="cuda"), n=0)
