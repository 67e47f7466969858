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

_u32p = ctypes.POINTER(ctypes.c_uint32)


def build_oracle() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE), "libngp_oracle.so"], check=True)
    return ORACLE_SO


def build_ref() -> Path | None:
    """Build oracle/_ref from the reference sources when they are present (not on a GPU box)."""
    if not Path("/root/reference/ngp.train.cu").exists():
        return REF_SO if REF_SO.exists() else None
    subprocess.run(["make", "-s", "-C", str(HERE), "ref"], check=True)
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

    def mlp_backward(self, params, x, coords, dy):
        params = np.ascontiguousarray(params.view(np.uint16))
        x = np.ascontiguousarray(x.view(np.uint16))
        dy = np.ascontiguousarray(dy.view(np.uint16))
        coords = np.ascontiguousarray(coords, np.float32)
        n = coords.shape[0]
        dx = np.zeros((32, n), np.uint16)
        dw = np.zeros(10240, np.float64)
        self.lib.oracle_mlp_backward(ctypes.c_uint32(n), _p(params), _p(x), ctypes.c_uint32(x.shape[1]), _p(coords),
                                     ctypes.c_uint32(coords.shape[1]), _p(dy), _p(dx), ctypes.c_uint32(n), _p(dw))
        return dx.view(np.float16), dw

    for f in (sh_encode, mlp_forward, density_forward, mlp_backward):
        setattr(Oracle, f.__name__, f)


_oracle_mlp_methods()
