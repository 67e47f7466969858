"""Python host binding of the B200-native NeRF hot path (``libngp_b200.so``).

This mirrors the reference's device-layer interface (``ngp::cuda`` in ngp.train.h:107-161):
the same operations, argument meanings and error behaviour (a failed call raises
``RuntimeError`` carrying the library's message, as the reference throws
``std::runtime_error``).  Device buffers are torch CUDA tensors, used only as memory and streams;
every computation runs in the library's own sm_100a kernels through its C ABI
(``include/ngp_b200.h``).  There is no CPU fallback: importing this module on a machine without
the built library raises.
"""
from __future__ import annotations

import ctypes
import math
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "libngp_b200.so"

MAX_LEVELS = 32
SAMPLE_FLOATS = 7
RAY_FLOATS = 6


class GridLayout(ctypes.Structure):
    """ctypes mirror of ``ngp_grid_layout``."""

    _fields_ = [
        ("n_levels", ctypes.c_uint32),
        ("features_per_level", ctypes.c_uint32),
        ("log2_hashmap_size", ctypes.c_uint32),
        ("base_resolution", ctypes.c_uint32),
        ("log2_per_level_scale", ctypes.c_double),
        ("offsets", ctypes.c_uint32 * (MAX_LEVELS + 1)),
        ("resolution", ctypes.c_uint32 * MAX_LEVELS),
        ("scale", ctypes.c_float * MAX_LEVELS),
        ("n_entries", ctypes.c_uint32),
        ("n_params", ctypes.c_uint32),
    ]

    def level_offsets(self) -> list[int]:
        return [int(self.offsets[i]) for i in range(self.n_levels + 1)]

    def level_resolutions(self) -> list[int]:
        return [int(self.resolution[i]) for i in range(self.n_levels)]

    def level_scales(self) -> list[float]:
        return [float(self.scale[i]) for i in range(self.n_levels)]


_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """Load the in-tree library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python instant-ngp_b200/build.py`")
        _lib = ctypes.CDLL(str(LIB_PATH))
        _lib.ngp_last_error.restype = ctypes.c_char_p
        _lib.ngp_version.restype = ctypes.c_char_p
    return _lib


def _check(status: int, what: str) -> None:
    if status != 0:
        msg = lib().ngp_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed (status {status}): {msg}")


def _ptr(t) -> ctypes.c_void_p:
    """Device pointer of a torch tensor (or None)."""
    if t is None:
        return ctypes.c_void_p(0)
    return ctypes.c_void_p(t.data_ptr())


def _stream(stream) -> ctypes.c_void_p:
    if stream is None:
        import torch

        return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if isinstance(stream, int):
        return ctypes.c_void_p(stream)
    return ctypes.c_void_p(stream.cuda_stream)


def version() -> str:
    return lib().ngp_version().decode()


def grid_layout(n_levels: int = 8, features_per_level: int = 4, log2_hashmap_size: int = 19, base_resolution: int = 16,
                log2_per_level_scale: float = 1.0) -> GridLayout:
    """Hash-grid layout; the defaults are the reference's (ngp.train.h:11-15)."""
    out = GridLayout()
    _check(lib().ngp_grid_layout_make(ctypes.c_uint32(n_levels), ctypes.c_uint32(features_per_level),
                                      ctypes.c_uint32(log2_hashmap_size), ctypes.c_uint32(base_resolution),
                                      ctypes.c_double(log2_per_level_scale), ctypes.byref(out)), "ngp_grid_layout_make")
    return out


def config0_layout() -> GridLayout:
    """L=16, F=2, log2 T=19, base 16, b = exp(ln(2048/16)/15)."""
    return grid_layout(16, 2, 19, 16, math.log2(2048.0 / 16.0) / 15.0)


def encode_grid_forward(layout: GridLayout, coords, table, out, n: int | None = None, coord_stride: int | None = None,
                        out_stride: int | None = None, stream=None) -> None:
    """Hash-grid forward (replaces encode_grid_forward_kernel, ngp.train.cu:876-921)."""
    n = coords.shape[0] if n is None else n
    coord_stride = coords.shape[1] if coord_stride is None else coord_stride
    out_stride = out.shape[1] if out_stride is None else out_stride
    _check(lib().ngp_encode_grid_forward(ctypes.byref(layout), ctypes.c_uint32(n), _ptr(coords), ctypes.c_uint32(coord_stride),
                                         _ptr(table), _ptr(out), ctypes.c_uint32(out_stride), _stream(stream)),
           "ngp_encode_grid_forward")


def encode_grid_backward(layout: GridLayout, coords, dy, table_grad, n: int | None = None, coord_stride: int | None = None,
                         dy_stride: int | None = None, stream=None) -> None:
    """Hash-grid backward into an fp32 gradient table (replaces encode_grid_backward_kernel, ngp.train.cu:923-960)."""
    n = coords.shape[0] if n is None else n
    coord_stride = coords.shape[1] if coord_stride is None else coord_stride
    dy_stride = dy.shape[1] if dy_stride is None else dy_stride
    _check(lib().ngp_encode_grid_backward(ctypes.byref(layout), ctypes.c_uint32(n), _ptr(coords), ctypes.c_uint32(coord_stride),
                                          _ptr(dy), ctypes.c_uint32(dy_stride), _ptr(table_grad), _stream(stream)),
           "ngp_encode_grid_backward")


# ---------------------------------------------------------------------------------------------
# Fully fused MLPs (replaces mlp_forward_64_relu_kernel / backward + cuBLASLt, ngp.train.cu:1019-1903)
# ---------------------------------------------------------------------------------------------
MLP_PARAMS = 10240
_scratch = {}


def sh_encode(coords, out, n: int | None = None, out_stride: int | None = None, stream=None) -> None:
    """Degree-4 SH of the sample records' view directions -> fp16 [16][out_stride]."""
    n = coords.shape[0] if n is None else n
    out_stride = out.shape[1] if out_stride is None else out_stride
    _check(lib().ngp_sh_encode(ctypes.c_uint32(n), _ptr(coords), ctypes.c_uint32(coords.shape[1]), _ptr(out),
                               ctypes.c_uint32(out_stride), _stream(stream)), "ngp_sh_encode")


def mlp_forward(params, x, coords, out, n: int | None = None, x_stride: int | None = None, density_rgb_in=None, stream=None) -> None:
    """Density + colour network forward -> out fp16 [n][16]."""
    n = coords.shape[0] if n is None else n
    x_stride = x.shape[1] if x_stride is None else x_stride
    _check(lib().ngp_mlp_forward(ctypes.c_uint32(n), _ptr(params), _ptr(x), ctypes.c_uint32(x_stride), _ptr(coords),
                                 ctypes.c_uint32(coords.shape[1]), _ptr(out), _ptr(density_rgb_in), _stream(stream)), "ngp_mlp_forward")


def density_forward(params, x, out, n: int | None = None, x_stride: int | None = None, stream=None) -> None:
    """Density network only -> raw density fp16 [n]."""
    n = out.shape[0] if n is None else n
    x_stride = x.shape[1] if x_stride is None else x_stride
    _check(lib().ngp_density_forward(ctypes.c_uint32(n), _ptr(params), _ptr(x), ctypes.c_uint32(x_stride), _ptr(out), _stream(stream)),
           "ngp_density_forward")


def mlp_backward_scratch(device=None):
    """The (cached) fp32 scratch buffer ngp_mlp_backward needs on `device`."""
    import torch

    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if dev not in _scratch:
        lib().ngp_mlp_backward_scratch_floats.restype = ctypes.c_uint32
        _scratch[dev] = torch.empty(int(lib().ngp_mlp_backward_scratch_floats()), dtype=torch.float32, device=dev)
    return _scratch[dev]


def mlp_backward(params, x, coords, dy, dx=None, dw_f32=None, dw_f16=None, dw_scale: float = 1.0, n: int | None = None,
                 x_stride: int | None = None, dx_stride: int | None = None, scratch=None, stream=None) -> None:
    """Network backward: dy fp16 [n][16] -> dx fp16 [32][dx_stride] and dw (scaled) fp32/fp16 [10240]."""
    n = coords.shape[0] if n is None else n
    x_stride = x.shape[1] if x_stride is None else x_stride
    if dx_stride is None:
        dx_stride = dx.shape[1] if dx is not None else n
    scratch = mlp_backward_scratch(x.device) if scratch is None else scratch
    _check(lib().ngp_mlp_backward(ctypes.c_uint32(n), _ptr(params), _ptr(x), ctypes.c_uint32(x_stride), _ptr(coords),
                                  ctypes.c_uint32(coords.shape[1]), _ptr(dy), _ptr(dx), ctypes.c_uint32(dx_stride), _ptr(scratch),
                                  ctypes.c_size_t(scratch.numel()), _ptr(dw_f32), _ptr(dw_f16), ctypes.c_float(dw_scale),
                                  _stream(stream)), "ngp_mlp_backward")


def mlp_status(reset: bool = False) -> int:
    v = ctypes.c_uint32(0)
    _check(lib().ngp_mlp_status(ctypes.byref(v), ctypes.c_int(1 if reset else 0)), "ngp_mlp_status")
    return int(v.value)
