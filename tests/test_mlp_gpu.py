"""Fused MLP parity (tcgen05 kernels) against the CPU oracle and the reference's WMMA kernels.

Tolerances (north_star: MLP outputs within 2e-3 relative):
* SH encoding, library vs oracle: bit-exact; library vs the reference kernel: <= 1 fp16 ulp.
* forward / backward, library vs oracle (same rounding points, fp32 accumulation; only the tensor
  core's summation order differs): |a - b| <= 2e-3 * |b| + 2e-3 * max|b|.
* forward, library (fp32 accumulation) vs reference (fp16 WMMA accumulation):
  max|a - b| <= 1e-2 * max|b| and mean|a - b| <= 2e-3 * max|b|.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import workloads

pytestmark = pytest.mark.gpu


def _t(a):
    import torch

    if a.dtype == np.float16:
        return torch.from_numpy(a).cuda()
    return torch.from_numpy(a).cuda()


def close(got, want, rtol=2e-3, atol_frac=2e-3):
    got = got.astype(np.float64)
    want = want.astype(np.float64)
    tol = rtol * np.abs(want) + atol_frac * np.abs(want).max()
    bad = np.abs(got - want) > tol
    return not bad.any(), float(np.abs(got - want).max() / max(np.abs(want).max(), 1e-30))


def test_sh_bit_exact_vs_oracle(ngp, oracle):
    import torch

    _, coords, _ = workloads.mlp_inputs(5000, seed=1)
    out = torch.zeros((16, 5000), dtype=torch.float16, device="cuda")
    ngp.sh_encode(_t(coords), out)
    torch.cuda.synchronize()
    assert out.cpu().numpy().view(np.uint16).tobytes() == oracle.sh_encode(coords).view(np.uint16).tobytes()


def test_sh_vs_reference(ngp, reflib):
    import torch

    n = 5000
    _, coords, _ = workloads.mlp_inputs(n, seed=2)
    ours = torch.zeros((16, n), dtype=torch.float16, device="cuda")
    ref = torch.zeros((16, n), dtype=torch.float16, device="cuda")
    c = _t(coords)
    ngp.sh_encode(c, ours)
    reflib.call("ref_sh_encode", ctypes.c_uint32(n), ctypes.c_void_p(c.data_ptr()), ctypes.c_void_p(ref.data_ptr()), ctypes.c_void_p(0))
    torch.cuda.synchronize()
    a = ours.cpu().numpy().view(np.int16).astype(np.int32)
    b = ref.cpu().numpy().view(np.int16).astype(np.int32)
    assert np.abs(a - b).max() <= 1  # adjacent fp16 encodings


@pytest.mark.parametrize("n", [1, 100, 128, 1000, 4096])
def test_forward_vs_oracle(ngp, oracle, n):
    import torch

    params = workloads.xavier_mlp_params(n)
    x, coords, _ = workloads.mlp_inputs(n, seed=n + 1)
    out = torch.zeros((n, 16), dtype=torch.float16, device="cuda")
    ngp.mlp_forward(_t(params), _t(x), _t(coords), out)
    torch.cuda.synchronize()
    assert ngp.mlp_status(reset=True) == 0
    ok, err = close(out.cpu().numpy(), oracle.mlp_forward(params, x, coords))
    assert ok, err


@pytest.mark.parametrize("n", [1, 300, 4096])
def test_density_forward_vs_oracle(ngp, oracle, n):
    import torch

    params = workloads.xavier_mlp_params(3)
    x, _, _ = workloads.mlp_inputs(n, seed=5)
    out = torch.zeros(n, dtype=torch.float16, device="cuda")
    ngp.density_forward(_t(params), _t(x), out)
    torch.cuda.synchronize()
    ok, err = close(out.cpu().numpy(), oracle.density_forward(params, x))
    assert ok, err


def test_forward_full_size_vs_oracle_sample(ngp, oracle):
    """2^18 rows (config 1); every 61st row checked against the oracle."""
    import torch

    n = 1 << 18
    params = workloads.xavier_mlp_params(7)
    x, coords, _ = workloads.mlp_inputs(n, seed=7)
    out = torch.zeros((n, 16), dtype=torch.float16, device="cuda")
    ngp.mlp_forward(_t(params), _t(x), _t(coords), out)
    torch.cuda.synchronize()
    idx = np.arange(0, n, 61)
    want = oracle.mlp_forward(params, np.ascontiguousarray(x[:, idx]), coords[idx])
    ok, err = close(out.cpu().numpy()[idx], want)
    assert ok, err


def test_forward_vs_reference_wmma(ngp, reflib):
    import torch

    n = 4096
    params = workloads.xavier_mlp_params(11)
    x, coords, _ = workloads.mlp_inputs(n, seed=11)
    P, X, C = _t(params), _t(x), _t(coords)
    ours = torch.zeros((n, 16), dtype=torch.float16, device="cuda")
    ngp.mlp_forward(P, X, C, ours)
    rgb_in = torch.zeros((32, n), dtype=torch.float16, device="cuda")
    ref_out = torch.zeros((n, 16), dtype=torch.float16, device="cuda")
    # the reference's rgb input rows 16..31 hold its own SH encoding of the directions
    reflib.call("ref_sh_encode", ctypes.c_uint32(n), ctypes.c_void_p(C.data_ptr()), ctypes.c_void_p(rgb_in[16:].data_ptr()), ctypes.c_void_p(0))
    reflib.call("ref_mlp_forward", ctypes.c_uint32(n), ctypes.c_void_p(P.data_ptr()), ctypes.c_void_p(X.data_ptr()),
                ctypes.c_void_p(rgb_in.data_ptr()), ctypes.c_void_p(ref_out.data_ptr()), ctypes.c_void_p(0))
    torch.cuda.synchronize()
    a = ours.float().cpu().numpy()[:, :4]
    b = ref_out.float().cpu().numpy()[:, :4]
    scale = np.abs(b).max()
    assert np.abs(a - b).max() <= 1e-2 * scale
    assert np.abs(a - b).mean() <= 2e-3 * scale


@pytest.mark.parametrize("n", [1, 128, 1000, 4096])
def test_backward_vs_oracle(ngp, oracle, n):
    import torch

    params = workloads.xavier_mlp_params(n + 2)
    x, coords, dy = workloads.mlp_inputs(n, seed=n + 3)
    dx = torch.zeros((32, n), dtype=torch.float16, device="cuda")
    dw = torch.zeros(10240, dtype=torch.float32, device="cuda")
    ngp.mlp_backward(_t(params), _t(x), _t(coords), _t(dy), dx=dx, dw_f32=dw)
    torch.cuda.synchronize()
    assert ngp.mlp_status(reset=True) == 0
    want_dx, want_dw = oracle.mlp_backward(params, x, coords, dy)
    ok, err = close(dx.cpu().numpy(), want_dx)
    assert ok, ("dx", err)
    got_dw = dw.cpu().numpy()
    for name, lo, hi in (("Wd_in", 0, 2048), ("Wd_out", 2048, 3072), ("Wr_in", 3072, 5120), ("Wr_h", 5120, 9216), ("Wr_out", 9216, 10240)):
        ok, err = close(got_dw[lo:hi], want_dw[lo:hi], rtol=5e-3, atol_frac=5e-3)
        assert ok, (name, err)


def test_backward_deterministic_and_scaled(ngp):
    import torch

    n = 1 << 16
    params = workloads.xavier_mlp_params(5)
    x, coords, dy = workloads.mlp_inputs(n, seed=6)
    P, X, C, DY = _t(params), _t(x), _t(coords), _t(dy)
    outs = []
    for scale in (1.0, 1.0, 0.5):
        dw = torch.zeros(10240, dtype=torch.float32, device="cuda")
        dw16 = torch.zeros(10240, dtype=torch.float16, device="cuda")
        ngp.mlp_backward(P, X, C, DY, dw_f32=dw, dw_f16=dw16, dw_scale=scale)
        torch.cuda.synchronize()
        outs.append((dw.cpu().numpy(), dw16.cpu().numpy()))
    assert outs[0][0].tobytes() == outs[1][0].tobytes()
    np.testing.assert_array_equal(outs[2][0], outs[0][0] * 0.5)
    assert (outs[0][1] == outs[0][0].astype(np.float16)).all()


def test_backward_full_size_vs_torch_fp32(ngp):
    """2^18 rows: gradients against a plain PyTorch fp32 restatement of the network that rounds to
    fp16 at the same points as the kernels (each layer output and each backpropagated gradient)."""
    import torch

    n = 1 << 18
    params = workloads.xavier_mlp_params(9)
    x, coords, dy = workloads.mlp_inputs(n, seed=9)
    P, X, C, DY = _t(params), _t(x), _t(coords), _t(dy)
    dw = torch.zeros(10240, dtype=torch.float32, device="cuda")
    dx = torch.zeros((32, n), dtype=torch.float16, device="cuda")
    ngp.mlp_backward(P, X, C, DY, dx=dx, dw_f32=dw)
    sh = torch.zeros((16, n), dtype=torch.float16, device="cuda")
    ngp.sh_encode(C, sh)
    torch.cuda.synchronize()

    def r(t):
        return t.half().float()

    W = [w.float().view(*s) for w, s in zip(torch.split(P, [2048, 1024, 2048, 4096, 1024]),
                                             [(64, 32), (16, 64), (64, 32), (64, 64), (16, 64)])]
    xin = X.float().T
    hd = r(torch.relu(xin @ W[0].T))
    do = r(hd @ W[1].T)
    ri = torch.cat([do, sh.float().T], dim=1)
    h1 = r(torch.relu(ri @ W[2].T))
    h2 = r(torch.relu(h1 @ W[3].T))
    g = DY.float()
    gy = torch.zeros((n, 16), device="cuda")
    gy[:, :3] = g[:, :3]
    dh2 = r(gy @ W[4]) * (h2 > 0)
    dh1 = r(dh2 @ W[3]) * (h1 > 0)
    dri = dh1 @ W[2]
    ddo = dri[:, :16].clone()
    ddo[:, 0] += g[:, 3]
    ddo = r(ddo)
    dhd = r(ddo @ W[1]) * (hd > 0)
    dxw = dhd @ W[0]
    want = torch.cat([(dhd.T @ xin).flatten(), (ddo.T @ hd).flatten(), (dh1.T @ ri).flatten(), (dh2.T @ h1).flatten(),
                      (gy.T @ h2).flatten()]).cpu().numpy()
    got = dw.cpu().numpy()
    for lo, hi in ((0, 2048), (2048, 3072), (3072, 5120), (5120, 9216), (9216, 10240)):
        err = np.abs(got[lo:hi] - want[lo:hi]).max() / np.abs(want[lo:hi]).max()
        assert err < 1e-2, (lo, err)
    dxw = dxw.T.cpu().numpy()
    # a hidden unit within one fp16 rounding of zero can flip its ReLU mask between the two
    # summation orders and change that row; all but a handful of rows must agree closely
    err = np.abs(dx.float().cpu().numpy() - dxw)
    scale = np.abs(dxw).max()
    assert (err <= 1e-2 * scale).mean() > 0.9999 and err.mean() <= 1e-4 * scale


@pytest.mark.parametrize("n", [8, 1000, 12206485])
def test_gradients_to_half_rounds_and_clears(ngp, n):
    """ngp_gradients_to_half (the conversion before the data-parallel exchange): fp16 rounding to
    nearest as torch's, the fp32 source zeroed, a tail past a multiple of 8 included."""
    import ctypes

    import torch

    g = torch.randn(n, dtype=torch.float32, device="cuda") * 100.0
    want = g.half()
    out = torch.zeros(n, dtype=torch.float16, device="cuda")
    rc = ngp.lib().ngp_gradients_to_half(ctypes.c_uint32(n), ctypes.c_void_p(g.data_ptr()), ctypes.c_void_p(out.data_ptr()), 1, None)
    torch.cuda.synchronize()
    assert rc == 0
    assert torch.equal(out.view(torch.int16), want.view(torch.int16))
    assert int(torch.count_nonzero(g)) == 0


@pytest.mark.parametrize("rows", [False, True], ids=["contiguous", "row-list"])
def test_density_forward_many_tiles_equals_full_network_channel(ngp, rows):
    """The density network alone at 2^20 rows (many tiles per CTA: the input ring and the
    register prefetch wrap around) equals channel 3 of the full network, bit for bit, for
    contiguous rows and for a row list."""
    import torch

    n = 1 << 20
    params = _t(workloads.xavier_mlp_params(7))
    x_h, c_h, _ = workloads.mlp_inputs(n, seed=17)
    x, coords = _t(x_h), _t(c_h)
    full = torch.zeros((n, 16), dtype=torch.float16, device="cuda")
    ngp.mlp_forward(params, x, coords, full)
    dens = torch.zeros(n, dtype=torch.float16, device="cuda")
    if rows:
        perm = torch.randperm(n, device="cuda", generator=torch.Generator(device="cuda").manual_seed(3)).to(torch.int32)
        cnt = torch.tensor([n], dtype=torch.int32, device="cuda")
        ngp.density_forward_rows(n, perm, cnt, params, x, n, dens)
    else:
        ngp.density_forward(params, x, dens)
    torch.cuda.synchronize()
    assert torch.equal(dens.view(torch.int16), full[:, 3].contiguous().view(torch.int16))
