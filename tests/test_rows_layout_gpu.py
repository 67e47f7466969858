"""Row-major encoded features (NGP_ROWS): the layout the trainer keeps its encodings in, so that
the network's input rows arrive by 16-byte asynchronous copies.  The same kernels, bit for bit:
the encoding writes the transpose of its feature-major output, and the networks' outputs, input
gradients and weight gradients from row-major inputs equal those from feature-major inputs
(dense and with row lists, ragged sizes included)."""
from __future__ import annotations

import math

import numpy as np
import pytest

import workloads

pytestmark = pytest.mark.gpu


def T(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("n", [1, 777, 1 << 16])
def test_encode_rows_is_the_transpose(ngp, n):
    import torch

    layout = ngp.grid_layout(16, 2, 19, 16, math.log2(128.0) / 15.0)
    coords, table, _ = workloads.encode_inputs(n, layout.n_params, 16, 2, seed=n, coord_stride=7)
    c, t = T(coords), T(table.view(np.int16))
    fm = torch.zeros((32, n), dtype=torch.float16, device="cuda")
    rm = torch.zeros((n, 32), dtype=torch.float16, device="cuda")
    ngp.encode_grid_forward(layout, c, t, fm)
    ngp.encode_grid_forward(layout, c, t, rm, out_stride=ngp.ROWS)
    # a row list: every third point, written at the point's own row
    rows = T(np.arange(0, n, 3, dtype=np.int32))
    rl = torch.zeros((n, 32), dtype=torch.float16, device="cuda")
    ngp.encode_grid_forward_rows(layout, rows.numel(), rows, None, c, t, rl, ngp.ROWS)
    torch.cuda.synchronize()
    assert torch.equal(rm, fm.t().contiguous())
    assert torch.equal(rl[::3], rm[::3]) and (n < 3 or bool((rl[1::3] == 0).all()))


@pytest.mark.parametrize("n", [1, 300, 4096, 50000])
def test_mlp_rows_equal_feature_major(ngp, n):
    import torch

    params = T(workloads.xavier_mlp_params(n).view(np.int16))
    x, coords, dy = workloads.mlp_inputs(n, seed=n + 3)
    xf, xr, c, g = T(x.view(np.int16)), T(np.ascontiguousarray(x.T).view(np.int16)), T(coords), T(dy.view(np.int16))
    out_f = torch.zeros((n, 16), dtype=torch.float16, device="cuda")
    out_r = torch.zeros_like(out_f)
    ngp.mlp_forward(params, xf, c, out_f)
    ngp.mlp_forward(params, xr, c, out_r, x_stride=ngp.ROWS)
    d_f = torch.zeros(n, dtype=torch.float16, device="cuda")
    d_r = torch.zeros_like(d_f)
    ngp.density_forward(params, xf, d_f)
    ngp.density_forward(params, xr, d_r, x_stride=ngp.ROWS)
    dx_f = torch.zeros((32, n), dtype=torch.float16, device="cuda")
    dx_r = torch.zeros_like(dx_f)
    dw_f = torch.zeros(10240, dtype=torch.float32, device="cuda")
    dw_r = torch.zeros_like(dw_f)
    ngp.mlp_backward(params, xf, c, g, dx=dx_f, dw_f32=dw_f)
    ngp.mlp_backward(params, xr, c, g, dx=dx_r, dw_f32=dw_r, x_stride=ngp.ROWS)
    torch.cuda.synchronize()
    assert ngp.mlp_status(reset=True) == 0
    assert torch.equal(out_f, out_r) and torch.equal(d_f, d_r)
    assert torch.equal(dx_f, dx_r) and torch.equal(dw_f, dw_r)


def test_mlp_rows_with_row_lists(ngp):
    """Row lists over row-major inputs (the trainer's batch): outputs at the listed samples'
    positions and gradients equal the feature-major run's."""
    import torch

    m, n = 70000, 20000
    rng = np.random.default_rng(9)
    rows_h = np.sort(rng.choice(m, n, replace=False)).astype(np.int32)
    params = T(workloads.xavier_mlp_params(2).view(np.int16))
    x, coords, dy = workloads.mlp_inputs(m, seed=21)
    xf, xr, c = T(x.view(np.int16)), T(np.ascontiguousarray(x.T).view(np.int16)), T(coords)
    rows, cnt = T(rows_h), T(np.array([n], np.int32))
    g = T(dy[:n].view(np.int16))
    o_f = torch.zeros((m, 16), dtype=torch.float16, device="cuda")
    o_r = torch.zeros_like(o_f)
    ngp.mlp_forward_rows(n + 100, rows, cnt, params, xf, m, c, o_f)
    ngp.mlp_forward_rows(n + 100, rows, cnt, params, xr, ngp.ROWS, c, o_r)
    den_f = torch.zeros(m, dtype=torch.float16, device="cuda")
    den_r = torch.zeros_like(den_f)
    ngp.density_forward_rows(n, rows, cnt, params, xf, m, den_f)
    ngp.density_forward_rows(n, rows, cnt, params, xr, ngp.ROWS, den_r)
    dx_f = torch.zeros((32, n), dtype=torch.float16, device="cuda")
    dx_r = torch.zeros_like(dx_f)
    dw_f = torch.zeros(10240, dtype=torch.float32, device="cuda")
    dw_r = torch.zeros_like(dw_f)
    ngp.mlp_backward_rows(n, rows, params, xf, m, c, g, dx_f, n, dw_f)
    ngp.mlp_backward_rows(n, rows, params, xr, ngp.ROWS, c, g, dx_r, n, dw_r)
    torch.cuda.synchronize()
    assert ngp.mlp_status(reset=True) == 0
    assert torch.equal(o_f, o_r) and torch.equal(den_f, den_r)
    assert torch.equal(dx_f, dx_r) and torch.equal(dw_f, dw_r)
    assert bool((o_r[rows.long()] != 0).any())
