"""Evaluation compositing and seeded initialisation: CUDA library vs the reference's own kernels
(oracle/_ref), the committed reference fixtures and the CPU oracle.

Bars:
* evaluation compositing (accumulate_evaluation_loss_kernel, ngp.train.cu:676-745): comparison
  image bytes equal to the reference kernel's (same fp32 operations and device math functions);
  fp64 SSE within 1e-9 relative (both sum the same per-pixel terms, in a different order);
  against the libm oracle within 1e-5 relative and 1 LSB;
* initialisation (initialize_mlp_parameters, initialize_grid_params_kernel): fp32 master and fp16
  parameters bit-equal to the reference's.
"""
from __future__ import annotations

import ctypes
import hashlib

import numpy as np
import pytest

import workloads
from conftest import GOLDEN

pytestmark = pytest.mark.gpu

V = ctypes.c_void_p


def T(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def P(t):
    return V(t.data_ptr())


def _ours(ngp, ns, co, out, px, image, W, H, offset, n):
    import torch

    sse = torch.zeros(1, dtype=torch.float64, device="cuda")
    comp = torch.zeros((H, 2 * W, 3), dtype=torch.uint8, device="cuda")
    rendered = torch.zeros((W * H, 3), dtype=torch.float32, device="cuda")
    ngp.eval_composite(n, offset, image, W, H, T(px), T(ns[offset:offset + n].astype(np.int32)), T(co), T(out.view(np.int16)), sse=sse,
                       comparison=comp, rendered=rendered, stream=0)
    torch.cuda.synchronize()
    return float(sse.item()), comp.cpu().numpy(), rendered.cpu().numpy()


def _reference(reflib, ns, co, out, px, image, W, H, offset, n):
    import torch

    sse = torch.zeros(1, dtype=torch.float64, device="cuda")
    comp = torch.zeros((H, 2 * W, 3), dtype=torch.uint8, device="cuda")
    keep = [T(px), T(ns[offset:offset + n].astype(np.int32)), T(co), T(out.view(np.int16))]
    reflib.call("ref_eval_composite", ctypes.c_uint32(n), ctypes.c_uint32(offset), ctypes.c_uint32(image), ctypes.c_uint32(W), ctypes.c_uint32(H),
                *[P(k) for k in keep], P(sse), P(comp))
    torch.cuda.synchronize()
    return float(sse.item()), comp.cpu().numpy()


@pytest.mark.parametrize("shape", [(64, 48, 0, None), (256, 192, 1000, 30000)], ids=["whole-image", "tile-at-offset"])
def test_eval_composite_matches_reference_kernel(ngp, reflib, oracle, shape):
    W, H, offset, n = shape
    ns, co, out, px = workloads.eval_composite_inputs(width=W, height=H, seed=91)
    n = W * H - offset if n is None else n
    sse, comp, rendered = _ours(ngp, ns, co, out, px, 1, W, H, offset, n)
    rsse, rcomp = _reference(reflib, ns, co, out, px, 1, W, H, offset, n)
    assert rsse > 0
    assert abs(sse - rsse) <= 1e-9 * rsse
    assert np.array_equal(comp, rcomp)
    # the rendered colours are the clamped composite whose bytes fill the comparison's right half
    pix = np.arange(offset, offset + n)
    right = rcomp.reshape(H, 2 * W, 3)[pix // W, W + pix % W]
    # (the kernel may fuse x * 255 + 0.5 into one rounding: allow 1 LSB)
    mine = (rendered[pix].astype(np.float64) * 255.0 + 0.5).astype(np.float32).astype(np.uint8)
    assert np.abs(mine.astype(np.int32) - right.astype(np.int32)).max() <= 1
    osse, ocomp = oracle.eval_composite(ns[offset:offset + n], co, out, px, 1, W, H, pixel_offset=offset, n=n)
    assert abs(osse - rsse) <= 1e-5 * rsse
    assert np.abs(ocomp.astype(np.int32) - rcomp.astype(np.int32)).max() <= 1


def test_eval_composite_matches_golden(ngp):
    g = np.load(GOLDEN / "eval_composite_ref.npz")
    ns, co, out, px = workloads.eval_composite_inputs(seed=int(g["seed"]))
    H, W = px.shape[1], px.shape[2]
    sse, comp, _ = _ours(ngp, ns, co, out, px, int(g["image"]), W, H, 0, W * H)
    assert abs(sse - float(g["sse"][0])) <= 1e-9 * float(g["sse"][0])
    assert np.array_equal(comp, g["comparison"])


def _init_ours(ngp, total):
    import torch

    master = torch.zeros(total, dtype=torch.float32, device="cuda")
    params = torch.zeros(total, dtype=torch.int16, device="cuda")
    ngp.init_mlp_parameters(master, params, stream=0)
    ngp.init_grid_parameters(total - 10240, master[10240:], params[10240:], stream=0)
    torch.cuda.synchronize()
    return master.cpu().numpy(), params.cpu().numpy().view(np.uint16)


def test_init_bit_exact_vs_reference(ngp, reflib):
    import torch

    total = int(reflib.lib.ref_total_param_count())
    master, params = _init_ours(ngp, total)
    rm = torch.zeros(total, dtype=torch.float32, device="cuda")
    rp = torch.zeros(total, dtype=torch.int16, device="cuda")
    rg = torch.zeros(total, dtype=torch.int16, device="cuda")
    reflib.call("ref_init_params", P(rm), P(rp), P(rg))
    torch.cuda.synchronize()
    assert master.tobytes() == rm.cpu().numpy().tobytes()
    assert params.tobytes() == rp.cpu().numpy().view(np.uint16).tobytes()


def test_init_matches_golden_and_config0_layout(ngp, oracle):
    g = np.load(GOLDEN / "init_ref.npz")
    master, params = _init_ours(ngp, int(g["total"]))
    assert hashlib.sha256(master.tobytes()).hexdigest() == str(g["master_sha256"])
    assert hashlib.sha256(params.tobytes()).hexdigest() == str(g["params_sha256"])
    # the config-0 layout (16 x 2, 12.2 M parameters) draws the same way: library == oracle
    n_grid = ngp.config0_layout().n_params
    m0, p0 = _init_ours(ngp, 10240 + n_grid)
    om, op = oracle.init_params(n_grid)
    assert m0.tobytes() == om.tobytes() and p0.tobytes() == op.tobytes()
