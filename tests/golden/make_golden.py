"""Generate the golden fixtures of this directory from the REFERENCE's own kernels.

Run on a machine with a GPU and oracle/_ref/libngp_ref.so (built from the reference sources by
`make -C oracle ref`):  python tests/golden/make_golden.py [fixture-name ...]
(no names: every fixture; names: only those files, e.g. eval_composite_ref.npz init_ref.npz);
NGP_GOLDEN_OUT names another output directory.
Inputs are regenerated deterministically from numpy seeds (workloads.py); only small inputs and
the reference's outputs are stored.  The CPU tests (tests/test_golden.py) check the CPU oracle
against these fixtures, which pins the oracle to the reference without a GPU.
"""
from __future__ import annotations

import ctypes
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path[:0] = [str(ROOT / "instant-ngp_b200"), str(ROOT / "oracle")]

import workloads  # noqa: E402
from oracle import RefLib  # noqa: E402


def main(only: set[str]) -> None:
    import torch

    out_dir = Path(os.environ.get("NGP_GOLDEN_OUT", str(HERE)))
    out_dir.mkdir(parents=True, exist_ok=True)

    def save(name, **arrays):
        if not only or name in only:
            np.savez_compressed(out_dir / name, **arrays)

    ref = RefLib()
    V = ctypes.c_void_p

    def P(t):
        return V(t.data_ptr())

    # PCG32 of the reference (host code)
    u, f = ref.pcg32(1337, 1, 12345, 64)
    save("pcg32_ref.npz", seed=1337, seq=1, advance=12345, uint=u, float=f)

    # encode_grid_forward_kernel, reference layout, 512 points
    n_grid = int(ref.lib.ref_total_param_count()) - int(ref.lib.ref_mlp_param_count())
    coords, table, _ = workloads.encode_inputs(512, n_grid, 8, 4, seed=2024, coord_stride=7)
    out = torch.zeros((32, 512), dtype=torch.float16, device="cuda")
    c, t = torch.from_numpy(coords).cuda(), torch.from_numpy(table.view(np.int16)).cuda()
    ref.call("ref_encode_forward", ctypes.c_uint32(512), P(c), P(t), P(out), V(0))
    torch.cuda.synchronize()
    save("encode_forward_ref.npz", n=512, n_grid=n_grid, seed=2024, out=out.cpu().numpy().view(np.uint16))

    # encode_spherical_harmonics_kernel, 512 directions
    _, mc, _ = workloads.mlp_inputs(512, seed=2025)
    sh = torch.zeros((16, 512), dtype=torch.float16, device="cuda")
    mct = torch.from_numpy(mc).cuda()  # kept alive until the kernel has run
    ref.call("ref_sh_encode", ctypes.c_uint32(512), P(mct), P(sh), V(0))
    torch.cuda.synchronize()
    save("sh_ref.npz", n=512, seed=2025, out=sh.cpu().numpy().view(np.uint16))

    # marching of config-2 rays through the Gaussian-blob occupancy grid (reference helpers)
    vals = workloads.blob_grid_values(workloads.gaussian_blob_density())
    bits = np.packbits((vals > 0.01).reshape(-1, 8), axis=1, bitorder="little").reshape(-1)
    rays = workloads.march_rays_config2(256, seed=2026)
    ns = torch.zeros(256, dtype=torch.int32, device="cuda")
    co = torch.zeros((256 * 1024, 7), dtype=torch.float32, device="cuda")
    rt, bt = torch.from_numpy(rays).cuda(), torch.from_numpy(bits).cuda()
    ref.call("ref_march_given_rays", ctypes.c_uint32(256), P(rt), P(bt), P(ns), P(co))
    torch.cuda.synchronize()
    ns_h = ns.cpu().numpy().astype(np.uint32)
    co_h = co.cpu().numpy().reshape(256, 1024, 7)
    packed = np.concatenate([co_h[i, :ns_h[i]] for i in range(256)]) if ns_h.sum() else np.zeros((0, 7), np.float32)
    save("march_ref.npz", n=256, seed=2026, numsteps=ns_h, coords=packed)

    # generate_density_grid_samples_kernel on the blob grid, 2048 uniform + 2048 non-uniform
    vt = torch.from_numpy(vals).cuda()
    gc = torch.zeros((4096, 7), dtype=torch.float32, device="cuda")
    gi = torch.zeros(4096, dtype=torch.int32, device="cuda")
    ref.call("ref_grid_samples", ctypes.c_uint32(2048), ctypes.c_uint32(2048), ctypes.c_uint32(3), P(vt), P(gc), P(gi))
    torch.cuda.synchronize()
    save("grid_samples_ref.npz", n_uniform=2048, n_nonuniform=2048, ema_step=3, coords=gc.cpu().numpy(),
                        indices=gi.cpu().numpy().astype(np.uint32))
    # accumulate_evaluation_loss_kernel on every pixel of image 1 (64 x 48), ragged sample runs
    ns_e, co_e, out_e, px_e = workloads.eval_composite_inputs(seed=2027)
    W, H = px_e.shape[2], px_e.shape[1]
    tns, tco, tout, tpx = (torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (ns_e.astype(np.int32), co_e, out_e.view(np.int16), px_e))
    sse = torch.zeros(1, dtype=torch.float64, device="cuda")
    comp = torch.zeros((H, 2 * W, 3), dtype=torch.uint8, device="cuda")
    ref.call("ref_eval_composite", ctypes.c_uint32(W * H), ctypes.c_uint32(0), ctypes.c_uint32(1), ctypes.c_uint32(W), ctypes.c_uint32(H), P(tpx),
             P(tns), P(tco), P(tout), P(sse), P(comp))
    torch.cuda.synchronize()
    save("eval_composite_ref.npz", seed=2027, image=1, sse=sse.cpu().numpy(), comparison=comp.cpu().numpy())

    # initialize_mlp_parameters + initialize_grid_parameters: MLP weights, a strided sample of the
    # grid entries and digests of the whole fp32 / fp16 vectors
    import hashlib

    total = int(ref.lib.ref_total_param_count())
    master = torch.zeros(total, dtype=torch.float32, device="cuda")
    params = torch.zeros(total, dtype=torch.int16, device="cuda")
    grads = torch.zeros(total, dtype=torch.int16, device="cuda")
    ref.call("ref_init_params", P(master), P(params), P(grads))
    torch.cuda.synchronize()
    m_h, p_h = master.cpu().numpy(), params.cpu().numpy().view(np.uint16)
    save("init_ref.npz", total=total, mlp=m_h[:10240], grid_stride=997, grid_sample=m_h[10240::997],
                        master_sha256=hashlib.sha256(m_h.tobytes()).hexdigest(), params_sha256=hashlib.sha256(p_h.tobytes()).hexdigest())
    print("golden fixtures written to", out_dir)


if __name__ == "__main__":
    main(set(sys.argv[1:]))
