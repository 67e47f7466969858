"""ctypes front end of the test oracles (TEST INFRASTRUCTURE ONLY).

* ``Oracle``   -- the CPU restatement in ngp_oracle.cpp (libngp_oracle.so), numpy in / out.
* ``RefLib``   -- the reference's own CUDA kernels built from its sources by ref_harness.cu
                  (_ref/libngp_ref.so); device pointers in / out, needs a GPU.

Only tests/, __graft_entry__.smoke() and bench.py's baseline legs use this module.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "libngp_oracle.so"
REF_SO = HERE / "_ref" / "libngp_ref.so"
SHIM_REPLAY_SO = HERE / "_ref" / "libngp_shim_replay.so"

_u32p = ctypes.POINTER(ctypes.c_uint32)


def reference_dir() -> Path | None:
    """The reference's source tree: $NGP_REFERENCE_DIR, else BASELINE.json's reference_path; None
    when neither names an existing tree (as on a GPU box, which uses the prebuilt _ref/)."""
    import json
    import os

    cand = os.environ.get("NGP_REFERENCE_DIR")
    if not cand:
        baseline = HERE.parent / "BASELINE.json"
        if baseline.exists():
            cand = json.loads(baseline.read_text()).get("reference_path")
    if cand and (Path(cand) / "ngp.train.cu").exists():
        return Path(cand)
    return None


def build_oracle() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE), "libngp_oracle.so"], check=True)
    return ORACLE_SO


def build_ref() -> Path | None:
    """Build oracle/_ref from the reference sources when they are present (not on a GPU box)."""
    ref = reference_dir()
    if ref is None:
        return REF_SO if REF_SO.exists() else None
    subprocess.run(["make", "-s", "-C", str(HERE), f"REF_DIR={ref}", "ref", "shim"], check=True)
    return REF_SO


def _p(a: np.ndarray | None) -> ctypes.c_void_p:
    if a is None:
        return ctypes.c_void_p(0)
    assert a.flags["C_CONTIGUOUS"]
    return ctypes.c_void_p(a.ctypes.data)


class Oracle:
    def __init__(self) -> None:
        if not ORACLE_SO.exists():
            build_oracle()
        self.lib = ctypes.CDLL(str(ORACLE_SO))
        self.lib.oracle_grid_index.restype = ctypes.c_uint32

    # -- layout ------------------------------------------------------------------------------
    def grid_layout(self, L: int, F: int, log2T: int, base: int, log2_scale: float):
        offsets = np.zeros(L + 1, np.uint32)
        res = np.zeros(L, np.uint32)
        scale = np.zeros(L, np.float32)
        self.lib.oracle_grid_layout(ctypes.c_uint32(L), ctypes.c_uint32(F), ctypes.c_uint32(log2T), ctypes.c_uint32(base),
                                    ctypes.c_double(log2_scale), _p(offsets), _p(res), _p(scale))
        return offsets, res, scale

    def grid_index(self, hashmap_size: int, res: int, x: int, y: int, z: int) -> int:
        return int(self.lib.oracle_grid_index(ctypes.c_uint32(hashmap_size), ctypes.c_uint32(res), ctypes.c_uint32(x),
                                              ctypes.c_uint32(y), ctypes.c_uint32(z)))

    # -- encoding ----------------------------------------------------------------------------
    def encode_forward(self, layout, coords: np.ndarray, table: np.ndarray, F: int, mode: int = 0, threads: int = 1) -> np.ndarray:
        offsets, res, scale = layout
        L = len(res)
        coords = np.ascontiguousarray(coords, np.float32)
        table = np.ascontiguousarray(table.view(np.uint16))
        n = coords.shape[0]
        out = np.zeros((L * F, n), np.uint16)
        self.lib.oracle_encode_forward(ctypes.c_uint32(L), ctypes.c_uint32(F), _p(offsets), _p(res), _p(scale), ctypes.c_uint32(n),
                                       _p(coords), ctypes.c_uint32(coords.shape[1]), _p(table), _p(out), ctypes.c_uint32(n),
                                       ctypes.c_int(mode), ctypes.c_int(threads))
        return out.view(np.float16)

    def encode_backward(self, layout, coords: np.ndarray, dy: np.ndarray, F: int, threads: int = 1) -> np.ndarray:
        offsets, res, scale = layout
        L = len(res)
        coords = np.ascontiguousarray(coords, np.float32)
        dy = np.ascontiguousarray(dy.view(np.uint16))
        n = coords.shape[0]
        grad = np.zeros(int(offsets[-1]) * F, np.float64)
        self.lib.oracle_encode_backward(ctypes.c_uint32(L), ctypes.c_uint32(F), _p(offsets), _p(res), _p(scale), ctypes.c_uint32(n),
                                        _p(coords), ctypes.c_uint32(coords.shape[1]), _p(dy), ctypes.c_uint32(dy.shape[1]), _p(grad),
                                        ctypes.c_int(threads))
        return grad

    def pcg32(self, initstate: int, initseq: int, advance: int, count: int):
        u = np.zeros(count, np.uint32)
        f = np.zeros(count, np.float32)
        self.lib.oracle_pcg32(ctypes.c_uint64(initstate), ctypes.c_uint64(initseq), ctypes.c_uint64(advance), ctypes.c_uint32(count),
                              _p(u), _p(f))
        return u, f


class RefLib:
    """The reference's kernels (compiled from its sources).  Raises if _ref was not built."""

    def __init__(self) -> None:
        if not REF_SO.exists():
            raise RuntimeError(f"{REF_SO} missing: run `make -C oracle ref` where the reference sources are present")
        self.lib = ctypes.CDLL(str(REF_SO))
        self.lib.ref_total_param_count.restype = ctypes.c_uint32
        self.lib.ref_mlp_param_count.restype = ctypes.c_uint32

    def grid_offsets(self) -> np.ndarray:
        out = np.zeros(9, np.uint32)
        self.lib.ref_grid_offsets(_p(out))
        return out

    def pcg32(self, initstate: int, initseq: int, advance: int, count: int):
        u = np.zeros(count, np.uint32)
        f = np.zeros(count, np.float32)
        self.lib.ref_pcg32(ctypes.c_uint64(initstate), ctypes.c_uint64(initseq), ctypes.c_uint64(advance), ctypes.c_uint32(count),
                           _p(u), _p(f))
        return u, f

    def call(self, name: str, *args) -> None:
        status = getattr(self.lib, name)(*args)
        if status != 0:
            raise RuntimeError(f"{name} failed with CUDA status {status}")


class ReplayTrainer:
    """The reference's training loop (InstantNGP::train, ngp.train.cpp:108-155, replayed through
    the ngp::cuda interface by train_replay.inc) on one implementation of that interface: the
    reference's own ngp.train.cu (REF_SO) or this library's drop-in layer (SHIM_REPLAY_SO)."""

    def __init__(self, so: Path, split_train: dict, split_test: dict | None = None) -> None:
        if not so.exists():
            raise RuntimeError(f"{so} missing: run `make -C oracle ref shim` where the reference sources are present")
        self.lib = ctypes.CDLL(str(so))
        self.lib.ref_train_create.restype = ctypes.c_void_p
        px, cam = np.ascontiguousarray(split_train["pixels"]), np.ascontiguousarray(split_train["camera"], np.float32)
        self._keep = [px, cam]
        tpx = tcam = None
        n_test = 0
        if split_test is not None:
            tpx, tcam = np.ascontiguousarray(split_test["pixels"]), np.ascontiguousarray(split_test["camera"], np.float32)
            n_test = tpx.shape[0]
            self._keep += [tpx, tcam]
        self.frames, self.height, self.width = px.shape[0], px.shape[1], px.shape[2]
        self.n_test = n_test
        (fx, fy), (cx, cy) = split_train["focal"], split_train["principal"]
        h = self.lib.ref_train_create(_p(px), ctypes.c_size_t(px.nbytes), _p(cam), ctypes.c_uint32(self.frames), ctypes.c_uint32(self.width),
                                      ctypes.c_uint32(self.height), ctypes.c_float(fx), ctypes.c_float(fy), ctypes.c_float(cx), ctypes.c_float(cy),
                                      _p(tpx), ctypes.c_size_t(0 if tpx is None else tpx.nbytes), _p(tcam), ctypes.c_uint32(n_test))
        if not h:
            raise RuntimeError("ref_train_create failed")
        self.handle = ctypes.c_void_p(h)

    def train(self, steps: int) -> dict:
        out = (ctypes.c_float * 4)()
        rc = self.lib.ref_train_steps(self.handle, ctypes.c_int32(steps), out)
        if rc != 0:
            raise RuntimeError(f"ref_train_steps failed ({rc})")
        return {"elapsed_ms": float(out[0]), "measured": int(out[1]), "measured_before": int(out[2]), "rays_per_batch": int(out[3])}

    def test_psnr(self) -> float:
        sse = ctypes.c_double(0)
        if self.lib.ref_train_test_sse(self.handle, ctypes.byref(sse)) != 0:
            raise RuntimeError("ref_train_test_sse failed")
        mse = sse.value / (self.n_test * self.width * self.height * 3.0)
        return -10.0 * np.log10(mse) if mse > 0 else float("inf")

    def close(self) -> None:
        if self.handle:
            self.lib.ref_train_destroy(self.handle)
            self.handle = None


def _oracle_mlp_methods():
    def sh_encode(self, coords):
        coords = np.ascontiguousarray(coords, np.float32)
        n = coords.shape[0]
        out = np.zeros((16, n), np.uint16)
        self.lib.oracle_sh_encode(ctypes.c_uint32(n), _p(coords), ctypes.c_uint32(coords.shape[1]), _p(out))
        return out.view(np.float16)

    def mlp_forward(self, params, x, coords, threads: int = 1):
        params = np.ascontiguousarray(params.view(np.uint16))
        x = np.ascontiguousarray(x.view(np.uint16))
        coords = np.ascontiguousarray(coords, np.float32)
        n = coords.shape[0]
        out = np.zeros((n, 16), np.uint16)
        self.lib.oracle_mlp_forward(ctypes.c_uint32(n), _p(params), _p(x), ctypes.c_uint32(x.shape[1]), _p(coords),
                                    ctypes.c_uint32(coords.shape[1]), _p(out), ctypes.c_int(threads))
        return out.view(np.float16)

    def density_forward(self, params, x):
        params = np.ascontiguousarray(params.view(np.uint16))
        x = np.ascontiguousarray(x.view(np.uint16))
        n = x.shape[1]
        out = np.zeros(n, np.uint16)
        self.lib.oracle_density_forward(ctypes.c_uint32(n), _p(params), _p(x), ctypes.c_uint32(x.shape[1]), _p(out))
        return out.view(np.float16)

    def mlp_backward(self, params, x, coords, dy, threads: int = 1):
        params = np.ascontiguousarray(params.view(np.uint16))
        x = np.ascontiguousarray(x.view(np.uint16))
        dy = np.ascontiguousarray(dy.view(np.uint16))
        coords = np.ascontiguousarray(coords, np.float32)
        n = coords.shape[0]
        dx = np.zeros((32, n), np.uint16)
        dw = np.zeros(10240, np.float64)
        if threads <= 1:
            self.lib.oracle_mlp_backward(ctypes.c_uint32(n), _p(params), _p(x), ctypes.c_uint32(x.shape[1]), _p(coords),
                                         ctypes.c_uint32(coords.shape[1]), _p(dy), _p(dx), ctypes.c_uint32(n), _p(dw))
        else:  # weight gradients summed per thread, then in thread order (CPU baseline timing)
            self.lib.oracle_mlp_backward_mt(ctypes.c_uint32(n), _p(params), _p(x), ctypes.c_uint32(x.shape[1]), _p(coords),
                                            ctypes.c_uint32(coords.shape[1]), _p(dy), _p(dx), ctypes.c_uint32(n), _p(dw), ctypes.c_int(threads))
        return dx.view(np.float16), dw

    for f in (sh_encode, mlp_forward, density_forward, mlp_backward):
        setattr(Oracle, f.__name__, f)


_oracle_mlp_methods()


def _oracle_sampler_methods():
    def march_rays(self, rays, bitfield, jitter=False, step=0, sample_limit=1 << 22):
        rays = np.ascontiguousarray(rays, np.float32)
        bits = np.ascontiguousarray(bitfield, np.uint8)
        n = rays.shape[0]
        numsteps = np.zeros((n, 2), np.uint32)
        coords = np.zeros((min(sample_limit, n * 1024), 7), np.float32)
        self.lib.oracle_march_rays.restype = ctypes.c_uint32
        total = self.lib.oracle_march_rays(ctypes.c_uint32(n), _p(rays), ctypes.c_int(int(jitter)), ctypes.c_uint32(step), _p(bits),
                                           ctypes.c_uint32(sample_limit), _p(numsteps), _p(coords))
        return numsteps, coords, int(total)

    def march_rays_mt(self, rays, bitfield, threads: int, sample_limit=1 << 22):
        """Evaluation-rule march (start tmin + dt/2) over `threads` host threads; same output as
        march_rays(jitter=False)."""
        rays = np.ascontiguousarray(rays, np.float32)
        bits = np.ascontiguousarray(bitfield, np.uint8)
        n = rays.shape[0]
        numsteps = np.zeros((n, 2), np.uint32)
        coords = np.zeros((min(sample_limit, n * 1024), 7), np.float32)
        self.lib.oracle_march_rays_mt.restype = ctypes.c_uint32
        total = self.lib.oracle_march_rays_mt(ctypes.c_uint32(n), _p(rays), _p(bits), ctypes.c_uint32(sample_limit), _p(numsteps), _p(coords),
                                              ctypes.c_int(threads))
        return numsteps, coords, int(total)

    def march_segment(self, rays, bitfield, cap, ray_list=None, t_state=None, marched=None):
        """One segment of the segmented evaluation march; returns (numsteps [k][2], records, t_out)."""
        rays = np.ascontiguousarray(rays, np.float32)
        bits = np.ascontiguousarray(bitfield, np.uint8)
        lst = None if ray_list is None else np.ascontiguousarray(ray_list, np.uint32)
        n = rays.shape[0] if lst is None else lst.size
        ts = None if t_state is None else np.ascontiguousarray(t_state, np.float32)
        mk = None if marched is None else np.ascontiguousarray(marched, np.uint32)
        numsteps = np.zeros((n, 2), np.uint32)
        coords = np.zeros((max(1, n * min(cap, 1024)), 7), np.float32)
        t_out = np.zeros(n, np.float32)
        self.lib.oracle_march_segment.restype = ctypes.c_uint32
        total = self.lib.oracle_march_segment(ctypes.c_uint32(n), None if lst is None else _p(lst), _p(rays), _p(bits),
                                              None if ts is None else _p(ts), None if mk is None else _p(mk), ctypes.c_uint32(cap),
                                              _p(numsteps), _p(coords), _p(t_out))
        return numsteps, coords[:total], t_out

    def eval_composite(self, numsteps, coords, network_output, pixels, image, width, height, pixel_offset=0, n=None, comparison=True):
        """Evaluation compositing of pixels [pixel_offset, pixel_offset + n) of `image`
        (accumulate_evaluation_loss_kernel): returns (sse, comparison [height][2*width][3] or None)."""
        numsteps = np.ascontiguousarray(numsteps, np.uint32)
        n = numsteps.shape[0] if n is None else n
        coords = np.ascontiguousarray(coords, np.float32)
        out = np.ascontiguousarray(network_output).view(np.uint16)
        pixels = np.ascontiguousarray(pixels, np.uint8)
        sse = np.zeros(1, np.float64)
        comp = np.zeros((height, 2 * width, 3), np.uint8) if comparison else None
        self.lib.oracle_eval_composite(ctypes.c_uint32(n), ctypes.c_uint32(pixel_offset), ctypes.c_uint32(image), ctypes.c_uint32(width),
                                       ctypes.c_uint32(height), _p(pixels), _p(numsteps), _p(coords), _p(out), _p(sse), _p(comp))
        return float(sse[0]), comp

    def init_params(self, n_grid: int):
        """Seeded initial parameters (initialize_mlp_parameters + initialize_grid_params_kernel):
        (fp32 master, fp16 params as uint16) of 10240 + n_grid entries."""
        master = np.zeros(10240 + n_grid, np.float32)
        params = np.zeros(10240 + n_grid, np.uint16)
        self.lib.oracle_init_params(ctypes.c_uint32(n_grid), _p(master), _p(params))
        return master, params

    def grid_samples(self, n_uniform, n_nonuniform, ema_step, values):
        values = np.ascontiguousarray(values, np.float32)
        n = n_uniform + n_nonuniform
        coords = np.zeros((n, 7), np.float32)
        idx = np.zeros(n, np.uint32)
        self.lib.oracle_grid_samples(ctypes.c_uint32(n_uniform), ctypes.c_uint32(n_nonuniform), ctypes.c_uint32(ema_step), _p(values), _p(coords),
                                     _p(idx))
        return coords, idx

    def grid_update(self, values, scratch, decay=0.95):
        values = np.array(values, np.float32)
        scratch = np.ascontiguousarray(scratch, np.float32)
        mean = np.zeros(1, np.float32)
        bits = np.zeros(values.size // 8, np.uint8)
        self.lib.oracle_grid_update.restype = ctypes.c_uint32
        cnt = self.lib.oracle_grid_update(_p(values), _p(scratch), ctypes.c_float(decay), _p(mean), _p(bits))
        return values, float(mean[0]), bits, int(cnt)

    def adam(self, n_mlp, master, params, grads, m, v, steps, lr=1e-2, b1=0.9, b2=0.99, eps=1e-15, l2=1e-6, loss_scale=128.0, threads: int = 1):
        arrs = [np.array(a) for a in (master, params.view(np.uint16), grads, m, v, steps)]
        self.lib.oracle_adam_mt(ctypes.c_uint32(arrs[0].size), ctypes.c_uint32(n_mlp), ctypes.c_float(lr), ctypes.c_float(b1), ctypes.c_float(b2),
                                ctypes.c_float(eps), ctypes.c_float(l2), ctypes.c_float(loss_scale), *[_p(a) for a in arrs], ctypes.c_int(threads))
        arrs[1] = arrs[1].view(np.float16)
        return [arrs[i] for i in (0, 1, 3, 4, 5)]

    for f in (march_rays, march_rays_mt, march_segment, eval_composite, init_params, grid_samples, grid_update, adam):
        setattr(Oracle, f.__name__, f)


_oracle_sampler_methods()
