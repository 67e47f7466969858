"""The allocation-free loss entry point (ngp_training_loss_and_compact_noalloc).

Callers that cannot allocate device memory while the loss runs (host callbacks, plugin hosts with
a fixed memory budget) use this variant; its scratch is a static device array.  This file is
collected last so that a run stopping at the first failure has already run every other test.  It
checks, through the C ABI, that two calls in a row give the same results as the entry point that
takes caller-provided scratch (after a call on other inputs, and at the size limit), and that
requests beyond the static limit are refused."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import workloads

pytestmark = pytest.mark.gpu


def _setup(ngp, n, bits=None, out_seed=0):
    import torch

    scene = workloads.procedural_dataset(n_train=4, n_test=1, width=96, height=80, seed=11)
    tr = scene["train"]
    F, H, W = tr["pixels"].shape[:3]
    (fx, fy), (cx, cy) = tr["focal"], tr["principal"]
    pix = torch.from_numpy(tr["pixels"]).cuda()
    cam = torch.from_numpy(tr["camera"]).cuda()
    if bits is None:
        bits = torch.full((128 ** 3 // 8,), 0xFF, dtype=torch.uint8, device="cuda")
    limit = 1 << 21
    coords = torch.zeros((limit, 7), dtype=torch.float32, device="cuda")
    ns = torch.zeros((n, 2), dtype=torch.int32, device="cuda")
    rays = torch.zeros((n, 6), dtype=torch.float32, device="cuda")
    ridx = torch.zeros(n, dtype=torch.int32, device="cuda")
    totals = torch.zeros(ngp.march_scratch_words(n), dtype=torch.int32, device="cuda")
    rc = torch.zeros(1, dtype=torch.int32, device="cuda")
    sc = torch.zeros(1, dtype=torch.int32, device="cuda")
    ngp.march_training_rays(cam, F, W, H, fx, fy, cx, cy, 2, n, limit, bits, coords, rays, ridx, ns, totals, rc, sc)
    rng = np.random.default_rng(out_seed)
    out = torch.from_numpy(rng.normal(0, 2, (limit, 16)).astype(np.float16)).cuda()
    return dict(pix=pix, F=F, W=W, H=H, coords=coords, ns=ns, rays=rays, ridx=ridx, rc=rc, out=out)


def _outputs(torch, n):
    return dict(cc=torch.zeros(1, dtype=torch.int32, device="cuda"), ccoords=torch.zeros((1 << 18, 7), dtype=torch.float32, device="cuda"),
                dloss=torch.zeros((1 << 18, 16), dtype=torch.float16, device="cuda"), loss=torch.zeros(n, dtype=torch.float32, device="cuda"))


def _call_noalloc(ngp, s, o, ns, n):
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    return ngp.lib().ngp_training_loss_and_compact_noalloc(
        ctypes.c_uint32(n), ctypes.c_uint32(2), P(s["rc"]), P(s["pix"]), ctypes.c_uint32(s["F"]), ctypes.c_uint32(s["W"]), ctypes.c_uint32(s["H"]),
        P(s["out"]), P(o["cc"]), P(s["ridx"]), P(s["rays"]), P(ns), P(s["coords"]), P(o["ccoords"]), P(o["dloss"]), P(o["loss"]), ctypes.c_void_p(0))


def _call_with_scratch(ngp, torch, s, n):
    ref = _outputs(torch, n)
    ns_ref = s["ns"].clone()
    scratch = torch.zeros(ngp.loss_scratch_bytes(n), dtype=torch.uint8, device="cuda")
    ngp.training_loss_and_compact(n, 2, s["rc"], s["pix"], s["F"], s["W"], s["H"], s["out"], ref["cc"], s["ridx"], s["rays"], ns_ref, s["coords"],
                                  ref["ccoords"], ref["dloss"], ref["loss"], scratch, stream=0)
    torch.cuda.synchronize()
    return ref, ns_ref


def _assert_same(torch, o, ns, ref, ns_ref):
    """Same code on the same inputs with different scratch memory: bit-identical outputs."""
    assert int(o["cc"].item()) == int(ref["cc"].item()) > 0
    assert torch.equal(ns, ns_ref)
    assert torch.equal(o["ccoords"], ref["ccoords"])
    assert torch.equal(o["loss"], ref["loss"])
    assert torch.equal(o["dloss"], ref["dloss"])


def test_noalloc_matches_scratch_entry_point_twice(ngp):
    import torch

    n = 3000
    # a first call on other inputs and more rays leaves its own values in the static array, so the
    # calls compared below would show any scratch word that they read without writing it first
    other = _setup(ngp, 5000, out_seed=7)
    o = _outputs(torch, 5000)
    assert _call_noalloc(ngp, other, o, other["ns"].clone(), 5000) == 0, ngp.lib().ngp_last_error()
    torch.cuda.synchronize()
    s = _setup(ngp, n)
    ref, ns_ref = _call_with_scratch(ngp, torch, s, n)
    for _ in range(2):  # two calls in a row share (and reuse) the static scratch
        o = _outputs(torch, n)
        ns = s["ns"].clone()
        assert _call_noalloc(ngp, s, o, ns, n) == 0, ngp.lib().ngp_last_error()
        torch.cuda.synchronize()
        _assert_same(torch, o, ns, ref, ns_ref)


def test_noalloc_at_the_size_limit(ngp):
    """rays_per_batch equal to the limit: the static array is used to its last byte."""
    import torch

    lib = ngp.lib()
    lib.ngp_training_loss_and_compact_noalloc_max_rays.restype = ctypes.c_uint32
    n = int(lib.ngp_training_loss_and_compact_noalloc_max_rays())
    bits = torch.zeros(128 ** 3 // 8, dtype=torch.uint8, device="cuda")
    bits[::4096] = 0xFF  # scattered occupied cells: few samples per ray
    s = _setup(ngp, n, bits=bits, out_seed=3)
    ref, ns_ref = _call_with_scratch(ngp, torch, s, n)
    for _ in range(2):
        o = _outputs(torch, n)
        ns = s["ns"].clone()
        assert _call_noalloc(ngp, s, o, ns, n) == 0, lib.ngp_last_error()
        torch.cuda.synchronize()
        _assert_same(torch, o, ns, ref, ns_ref)


def test_noalloc_rejects_sizes_beyond_the_limit(ngp):
    import torch

    lib = ngp.lib()
    lib.ngp_training_loss_and_compact_noalloc_max_rays.restype = ctypes.c_uint32
    limit = int(lib.ngp_training_loss_and_compact_noalloc_max_rays())
    assert limit == 1 << 18
    s = _setup(ngp, 128)
    o = _outputs(torch, 128)
    assert _call_noalloc(ngp, s, o, s["ns"], limit + 1) == 1  # NGP_ERR_INVALID
    assert b"static scratch limit" in lib.ngp_last_error()
