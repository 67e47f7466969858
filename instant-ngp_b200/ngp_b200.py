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
import os
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ["NGP_B200_LIB"]) if os.environ.get("NGP_B200_LIB") else PKG_DIR / "libngp_b200.so"

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


def adaptive_batch(rays_per_batch: int, measured_before: int, measured: int) -> tuple[int, int]:
    """(next rays per batch, next inference sample count) of the adaptive batch rule."""
    r, i = ctypes.c_uint32(0), ctypes.c_uint32(0)
    lib().ngp_adaptive_batch(_u32(rays_per_batch), _u32(measured_before), _u32(measured), ctypes.byref(r), ctypes.byref(i))
    return int(r.value), int(i.value)


def kernel_launch_count() -> int:
    """Kernel launches made by the library in this process so far."""
    lib().ngp_kernel_launch_count.restype = ctypes.c_uint64
    return int(lib().ngp_kernel_launch_count())


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


def density_forward_splat(params, x, indices, scratch, n: int | None = None, x_stride: int | None = None, stream=None) -> None:
    """Density network + the density-grid splat into scratch[indices[i]] (atomic max)."""
    n = indices.shape[0] if n is None else n
    x_stride = x.shape[1] if x_stride is None else x_stride
    _check(lib().ngp_density_forward_splat(ctypes.c_uint32(n), _ptr(params), _ptr(x), ctypes.c_uint32(x_stride), _ptr(indices), _ptr(scratch),
                                           _stream(stream)), "ngp_density_forward_splat")


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


# ---------------------------------------------------------------------------------------------
# Occupancy grid, marching, compositing / loss, Adam (ngp.train.cu:310-874, 1261-1280)
# ---------------------------------------------------------------------------------------------
GRID_CELLS = 128 ** 3
NETWORK_BATCH = 1 << 18
ROWS = 0x80000000  # NGP_ROWS: pass as a feature-buffer stride for row-major [rows][features] buffers
MAX_SAMPLES = NETWORK_BATCH * 16


def _u32(v):
    return ctypes.c_uint32(int(v))


def _f32(v):
    return ctypes.c_float(float(v))


def density_grid_mark_untrained(camera, frame_count, width, height, fx, fy, cx, cy, values, stream=None) -> None:
    _check(lib().ngp_density_grid_mark_untrained(_ptr(camera), _u32(frame_count), _u32(width), _u32(height), _f32(fx), _f32(fy), _f32(cx),
                                                 _f32(cy), _ptr(values), _stream(stream)), "ngp_density_grid_mark_untrained")


def density_grid_samples(n_uniform, n_nonuniform, ema_step, values, coords, indices, stream=None) -> None:
    _check(lib().ngp_density_grid_samples(_u32(n_uniform), _u32(n_nonuniform), _u32(ema_step), _ptr(values), _ptr(coords), _ptr(indices),
                                          _stream(stream)), "ngp_density_grid_samples")


def density_grid_samples_cell_order(n_uniform, n_nonuniform, ema_step, values, coords, indices, counter=None, stream=None) -> None:
    _check(lib().ngp_density_grid_samples_cell_order(_u32(n_uniform), _u32(n_nonuniform), _u32(ema_step), _ptr(values), _ptr(coords), _ptr(indices),
                                                     _ptr(counter), _stream(stream)), "ngp_density_grid_samples_cell_order")


def density_grid_encode_samples(layout: GridLayout, ema_step, values, table, out, indices, out_stride=None, stream=None) -> None:
    """Warm-up grid samples generated and encoded in one pass (no positions written)."""
    out_stride = out.shape[1] if out_stride is None else out_stride
    _check(lib().ngp_density_grid_encode_samples(ctypes.byref(layout), _u32(ema_step), _ptr(values), _ptr(table), _ptr(out), _u32(out_stride),
                                                 _ptr(indices), _stream(stream)), "ngp_density_grid_encode_samples")


def density_grid_splat(n, indices, density, scratch, stream=None) -> None:
    _check(lib().ngp_density_grid_splat(_u32(n), _ptr(indices), _ptr(density), _ptr(scratch), _stream(stream)), "ngp_density_grid_splat")


def density_grid_update(values, scratch, partial, mean, bitfield, occupied, decay=0.95, stream=None) -> None:
    _check(lib().ngp_density_grid_update(_ptr(values), _ptr(scratch), _f32(decay), _ptr(partial), _ptr(mean), _ptr(bitfield), _ptr(occupied),
                                         _stream(stream)), "ngp_density_grid_update")


def density_grid_partials() -> int:
    lib().ngp_density_grid_partials.restype = ctypes.c_uint32
    return int(lib().ngp_density_grid_partials())


def march_scratch_words(max_rays: int) -> int:
    lib().ngp_march_scratch_words.restype = ctypes.c_uint64
    return int(lib().ngp_march_scratch_words(_u32(max_rays)))


def march_training_rays(camera, frame_count, width, height, fx, fy, cx, cy, step, rays_per_batch, sample_limit, bitfield, coords, rays,
                        ray_indices, numsteps, scratch, ray_counter, sample_counter, rays_per_batch_dev=None, stream=None) -> None:
    _check(lib().ngp_march_training_rays(_ptr(camera), _u32(frame_count), _u32(width), _u32(height), _f32(fx), _f32(fy), _f32(cx), _f32(cy),
                                         _u32(step), _u32(rays_per_batch), _ptr(rays_per_batch_dev), _u32(sample_limit), _ptr(bitfield),
                                         _ptr(coords), _ptr(rays), _ptr(ray_indices), _ptr(numsteps), _ptr(scratch), _ptr(ray_counter),
                                         _ptr(sample_counter), _stream(stream)), "ngp_march_training_rays")


def march_rays(rays, bitfield, coords, numsteps, scratch, sample_counter, sample_limit=MAX_SAMPLES, jitter=False, step=0, n=None,
               stream=None) -> None:
    n = rays.shape[0] if n is None else n
    _check(lib().ngp_march_rays(_u32(n), _ptr(rays), ctypes.c_int(1 if jitter else 0), _u32(step), _ptr(bitfield), _u32(sample_limit), _ptr(coords),
                                _ptr(numsteps), _ptr(scratch), _ptr(sample_counter), _stream(stream)), "ngp_march_rays")


def march_rays_segment(rays, bitfield, coords, numsteps, t_out, scratch, counters, cap, max_entries=None, n_entries=None, ray_list=None,
                       t_state=None, marched=None, sample_limit=MAX_SAMPLES, stream=None) -> None:
    max_entries = rays.shape[0] if max_entries is None else max_entries
    _check(lib().ngp_march_rays_segment(_u32(max_entries), _ptr(n_entries), _ptr(ray_list), _ptr(rays), _ptr(bitfield), _ptr(t_state), _ptr(marched),
                                        _u32(cap), _u32(sample_limit), _ptr(coords), _ptr(numsteps), _ptr(t_out), _ptr(scratch), _ptr(counters),
                                        _stream(stream)), "ngp_march_rays_segment")


def eval_composite_segment(max_entries, complete, numsteps, coords, network_output, t_out, t_state, marched, state, next_list, next_count,
                           pixel_offset, image, width, height, n_entries=None, ray_list=None, pixels=None, sse=None, comparison=None,
                           rendered=None, stream=None) -> None:
    _check(lib().ngp_eval_composite_segment(_u32(max_entries), _ptr(n_entries), _ptr(complete), _ptr(ray_list), _ptr(numsteps), _ptr(coords),
                                            _ptr(network_output), _ptr(t_out), _ptr(t_state), _ptr(marched), _ptr(state), _ptr(next_list),
                                            _ptr(next_count), _u32(pixel_offset), _u32(image), _u32(width), _u32(height), _ptr(pixels), _ptr(sse),
                                            _ptr(comparison), _ptr(rendered), _stream(stream)), "ngp_eval_composite_segment")


def make_eval_rays(camera, image, width, height, fx, fy, cx, cy, pixel_offset, n, rays, stream=None) -> None:
    _check(lib().ngp_make_eval_rays(_ptr(camera), _u32(image), _u32(width), _u32(height), _f32(fx), _f32(fy), _f32(cx), _f32(cy),
                                    _u32(pixel_offset), _u32(n), _ptr(rays), _stream(stream)), "ngp_make_eval_rays")


def loss_scratch_bytes(max_rays: int) -> int:
    lib().ngp_loss_scratch_bytes.restype = ctypes.c_uint32
    n = int(lib().ngp_loss_scratch_bytes(_u32(max_rays)))
    if n == 0:
        raise RuntimeError(f"ngp_loss_scratch_bytes: {lib().ngp_last_error().decode()}")
    return n


def training_loss_and_compact(rays_per_batch, step, ray_counter, pixels, frame_count, width, height, network_output, compacted_counter,
                              ray_indices, rays, numsteps, coords, compacted_coords, dloss_doutput, loss_values, scratch, stream=None) -> None:
    _check(lib().ngp_training_loss_and_compact(_u32(rays_per_batch), _u32(step), _ptr(ray_counter), _ptr(pixels), _u32(frame_count), _u32(width),
                                               _u32(height), _ptr(network_output), _ptr(compacted_counter), _ptr(ray_indices), _ptr(rays),
                                               _ptr(numsteps), _ptr(coords), _ptr(compacted_coords), _ptr(dloss_doutput), _ptr(loss_values),
                                               _ptr(scratch), ctypes.c_size_t(scratch.numel() * scratch.element_size()), _stream(stream)),
           "ngp_training_loss_and_compact")


def pad_training_batch(compacted_counter, compacted_coords, dloss_doutput, stream=None) -> None:
    _check(lib().ngp_pad_training_batch(_ptr(compacted_counter), _ptr(compacted_coords), _ptr(dloss_doutput), _stream(stream)),
           "ngp_pad_training_batch")


def compacted_rows() -> int:
    lib().ngp_compacted_rows.restype = ctypes.c_uint32
    return int(lib().ngp_compacted_rows())


def training_compact_by_density(rays_per_batch, ray_counter, density, coords, numsteps, compacted_coords, compacted_counter, scratch,
                                enc=None, enc_stride=0, compacted_enc=None, stream=None) -> None:
    _check(lib().ngp_training_compact_by_density(_u32(rays_per_batch), _ptr(ray_counter), _ptr(density), _ptr(coords), _ptr(enc), _u32(enc_stride),
                                                 _ptr(numsteps), _ptr(compacted_coords), _ptr(compacted_enc), _ptr(compacted_counter),
                                                 _ptr(scratch), ctypes.c_size_t(scratch.numel() * scratch.element_size()), _stream(stream)),
           "ngp_training_compact_by_density")


def training_compact_progressive(rays_per_batch, ray_counter, layout, params, coords, sample_bound, numsteps, enc, density, rows,
                                 compacted_coords, compacted_enc, compacted_counter, scratch, enc_stride=None, stream=None) -> None:
    _check(lib().ngp_training_compact_progressive(_u32(rays_per_batch), _ptr(ray_counter), ctypes.byref(layout), _ptr(params), _ptr(coords),
                                                  _u32(sample_bound), _ptr(numsteps), _ptr(enc), _u32(enc.shape[1] if enc_stride is None else enc_stride),
                                                  _ptr(density), _ptr(rows), _ptr(compacted_coords), _ptr(compacted_enc), _ptr(compacted_counter),
                                                  _ptr(scratch), ctypes.c_size_t(scratch.numel() * scratch.element_size()), _stream(stream)),
           "ngp_training_compact_progressive")


def eval_network_progressive(n_rays, layout, params, coords, sample_bound, numsteps, enc, network_output, rows, scratch, enc_stride=None,
                             stream=None) -> None:
    _check(lib().ngp_eval_network_progressive(_u32(n_rays), ctypes.byref(layout), _ptr(params), _ptr(coords), _u32(sample_bound), _ptr(numsteps),
                                              _ptr(enc), _u32(enc.shape[1] if enc_stride is None else enc_stride), _ptr(network_output),
                                              _ptr(rows), _ptr(scratch), ctypes.c_size_t(scratch.numel() * scratch.element_size()),
                                              _stream(stream)), "ngp_eval_network_progressive")


def training_select_progressive(rays_per_batch, ray_counter, layout, params, coords, sample_bound, numsteps, enc, density, rows, batch_rows,
                                n_selected, compacted_counter, scratch, enc_stride=None, stream=None) -> None:
    _check(lib().ngp_training_select_progressive(_u32(rays_per_batch), _ptr(ray_counter), ctypes.byref(layout), _ptr(params), _ptr(coords),
                                                 _u32(sample_bound), _ptr(numsteps), _ptr(enc), _u32(enc.shape[1] if enc_stride is None else enc_stride),
                                                 _ptr(density), _ptr(rows), _ptr(batch_rows), _ptr(n_selected), _ptr(compacted_counter), _ptr(scratch),
                                                 ctypes.c_size_t(scratch.numel() * scratch.element_size()), _stream(stream)),
           "ngp_training_select_progressive")


def training_select_progressive_window(rays_per_batch, ray_counter, layout, params, coords, sample_bound, numsteps, enc, density, rows, batch_rows,
                                       n_selected, compacted_counter, scratch, first_window, still_active=None, enc_stride=None,
                                       stream=None) -> None:
    """training_select_progressive with the first round's window (0xFFFFFFFF: one round)."""
    _check(lib().ngp_training_select_progressive_window(_u32(rays_per_batch), _ptr(ray_counter), ctypes.byref(layout), _ptr(params), _ptr(coords),
                                                        _u32(sample_bound), _ptr(numsteps), _ptr(enc),
                                                        _u32(enc.shape[1] if enc_stride is None else enc_stride), _ptr(density), _ptr(rows),
                                                        _ptr(batch_rows), _ptr(n_selected), _ptr(compacted_counter), _ptr(scratch),
                                                        ctypes.c_size_t(scratch.numel() * scratch.element_size()), _u32(first_window),
                                                        _ptr(still_active), _stream(stream)),
           "ngp_training_select_progressive_window")


def training_loss_selected_kind(rays_per_batch, step, ray_counter, pixels, frame_count, width, height, network_output, ray_indices, rays, numsteps,
                                coords, dloss, loss_values, scratch, loss_kind, stream=None) -> None:
    _check(lib().ngp_training_loss_selected_kind(_u32(rays_per_batch), _u32(step), _ptr(ray_counter), _ptr(pixels), _u32(frame_count), _u32(width),
                                                 _u32(height), _ptr(network_output), _ptr(ray_indices), _ptr(rays), _ptr(numsteps), _ptr(coords),
                                                 _ptr(dloss), _ptr(loss_values), _ptr(scratch), ctypes.c_size_t(scratch.numel() * scratch.element_size()),
                                                 ctypes.c_int(loss_kind), _stream(stream)), "ngp_training_loss_selected_kind")


def training_loss_selected(rays_per_batch, step, ray_counter, pixels, frame_count, width, height, network_output, ray_indices, rays, numsteps,
                           coords, dloss_doutput, loss_values, scratch, stream=None) -> None:
    _check(lib().ngp_training_loss_selected(_u32(rays_per_batch), _u32(step), _ptr(ray_counter), _ptr(pixels), _u32(frame_count), _u32(width),
                                            _u32(height), _ptr(network_output), _ptr(ray_indices), _ptr(rays), _ptr(numsteps), _ptr(coords),
                                            _ptr(dloss_doutput), _ptr(loss_values), _ptr(scratch),
                                            ctypes.c_size_t(scratch.numel() * scratch.element_size()), _stream(stream)), "ngp_training_loss_selected")


def pad_training_rows(compacted_counter, batch_rows, dloss_doutput, stream=None) -> None:
    _check(lib().ngp_pad_training_rows(_ptr(compacted_counter), _ptr(batch_rows), _ptr(dloss_doutput), _stream(stream)), "ngp_pad_training_rows")


def encode_grid_forward_rows(layout: GridLayout, max_rows, rows, n_rows, coords, table, out, out_stride, stream=None) -> None:
    _check(lib().ngp_encode_grid_forward_rows(ctypes.byref(layout), _u32(max_rows), _ptr(rows), _ptr(n_rows), _ptr(coords), _u32(coords.shape[1]),
                                              _ptr(table), _ptr(out), _u32(out_stride), _stream(stream)), "ngp_encode_grid_forward_rows")


def density_forward_rows(max_rows, rows, n_rows, params, x, x_stride, out, stream=None) -> None:
    _check(lib().ngp_density_forward_rows(_u32(max_rows), _ptr(rows), _ptr(n_rows), _ptr(params), _ptr(x), _u32(x_stride), _ptr(out),
                                          _stream(stream)), "ngp_density_forward_rows")


def mlp_forward_rows(max_rows, rows, n_rows, params, x, x_stride, coords, out, stream=None) -> None:
    _check(lib().ngp_mlp_forward_rows(_u32(max_rows), _ptr(rows), _ptr(n_rows), _ptr(params), _ptr(x), _u32(x_stride), _ptr(coords),
                                      _u32(coords.shape[1]), _ptr(out), _stream(stream)), "ngp_mlp_forward_rows")


def mlp_backward_rows(n, rows, params, x, x_stride, coords, dy, dx, dx_stride, dw_f32, stream=None) -> None:
    sc = mlp_backward_scratch()
    _check(lib().ngp_mlp_backward_rows(_u32(n), _ptr(rows), _ptr(params), _ptr(x), _u32(x_stride), _ptr(coords), _u32(coords.shape[1]), _ptr(dy),
                                       _ptr(dx), _u32(dx_stride), _ptr(sc), ctypes.c_size_t(sc.numel()), _ptr(dw_f32), None, ctypes.c_float(1.0),
                                       _stream(stream)), "ngp_mlp_backward_rows")


def encode_grid_backward_rows(layout, n, rows, coords, dy, table_grad, dy_stride=None, stream=None) -> None:
    _check(lib().ngp_encode_grid_backward_rows(ctypes.byref(layout), _u32(n), _ptr(rows), _ptr(coords), _u32(coords.shape[1]), _ptr(dy),
                                               _u32(dy.shape[1] if dy_stride is None else dy_stride), _ptr(table_grad), _stream(stream)),
           "ngp_encode_grid_backward_rows")


def training_loss_compacted(rays_per_batch, step, ray_counter, pixels, frame_count, width, height, compacted_output, ray_indices, rays,
                            numsteps, compacted_coords, dloss_doutput, loss_values, scratch, stream=None) -> None:
    _check(lib().ngp_training_loss_compacted(_u32(rays_per_batch), _u32(step), _ptr(ray_counter), _ptr(pixels), _u32(frame_count), _u32(width),
                                             _u32(height), _ptr(compacted_output), _ptr(ray_indices), _ptr(rays), _ptr(numsteps),
                                             _ptr(compacted_coords), _ptr(dloss_doutput), _ptr(loss_values), _ptr(scratch),
                                             ctypes.c_size_t(scratch.numel() * scratch.element_size()), _stream(stream)),
           "ngp_training_loss_compacted")


def pad_training_batch_enc(compacted_counter, compacted_coords, dloss_doutput, enc, enc_stride, stream=None) -> None:
    _check(lib().ngp_pad_training_batch_enc(_ptr(compacted_counter), _ptr(compacted_coords), _ptr(dloss_doutput), _ptr(enc), _u32(enc_stride),
                                            _stream(stream)), "ngp_pad_training_batch_enc")


def eval_composite(n_pixels, pixel_offset, image, width, height, pixels, numsteps, coords, network_output, sse=None, comparison=None,
                   rendered=None, stream=None) -> None:
    _check(lib().ngp_eval_composite(_u32(n_pixels), _u32(pixel_offset), _u32(image), _u32(width), _u32(height), _ptr(pixels), _ptr(numsteps),
                                    _ptr(coords), _ptr(network_output), _ptr(sse), _ptr(comparison), _ptr(rendered), _stream(stream)),
           "ngp_eval_composite")


def init_mlp_parameters(master, params, stream=None) -> None:
    """Xavier-uniform MLP weights from PCG32(1337) into master[0:10240] / params[0:10240]
    (initialize_mlp_parameters, ngp.train.cu:1423-1461)."""
    _check(lib().ngp_init_mlp_parameters(_ptr(master), _ptr(params), _stream(stream)), "ngp_init_mlp_parameters")


def init_grid_parameters(n_grid, master_grid, params_grid, stream=None) -> None:
    """U(-1e-4, 1e-4) grid entries (initialize_grid_params_kernel, ngp.train.cu:1002-1017)."""
    _check(lib().ngp_init_grid_parameters(_u32(n_grid), _ptr(master_grid), _ptr(params_grid), _stream(stream)), "ngp_init_grid_parameters")


def adam_step(n_mlp, master, params, grads, m, v, steps, lr=1e-2, beta1=0.9, beta2=0.99, eps=1e-15, l2_reg=1e-6, loss_scale=128.0,
              clear_grid_gradients=True, stream=None) -> None:
    _check(lib().ngp_adam_step(_u32(master.numel()), _u32(n_mlp), _f32(lr), _f32(beta1), _f32(beta2), _f32(eps), _f32(l2_reg), _f32(loss_scale),
                               _ptr(master), _ptr(params), _ptr(grads), _ptr(m), _ptr(v), _ptr(steps), ctypes.c_int(1 if clear_grid_gradients else 0),
                               _stream(stream)), "ngp_adam_step")


def adam_lr_table(table, first, count, lr=1e-2, beta1=0.9, beta2=0.99, stream=None) -> None:
    _check(lib().ngp_adam_lr_table(_ptr(table), _u32(first), _u32(count), _f32(lr), _f32(beta1), _f32(beta2), _stream(stream)),
           "ngp_adam_lr_table")


def adam_step_table(n_mlp, master, params, grads, m, v, steps, lr_table, table_len, lr=1e-2, beta1=0.9, beta2=0.99, eps=1e-15, l2_reg=1e-6,
                    loss_scale=128.0, clear_grid_gradients=True, stream=None) -> None:
    _check(lib().ngp_adam_step_table(_u32(master.numel()), _u32(n_mlp), _f32(lr), _f32(beta1), _f32(beta2), _f32(eps), _f32(l2_reg),
                                     _f32(loss_scale), _ptr(master), _ptr(params), _ptr(grads), _ptr(m), _ptr(v), _ptr(steps),
                                     ctypes.c_int(1 if clear_grid_gradients else 0), _ptr(lr_table), _u32(table_len), _stream(stream)),
           "ngp_adam_step_table")


# ---------------------------------------------------------------------------------------------
# Trainer (the reference's ngp::train::InstantNGP, ngp.train.ixx:40-53)
# ---------------------------------------------------------------------------------------------
class TrainerConfig(ctypes.Structure):
    _fields_ = [("n_levels", ctypes.c_uint32), ("features_per_level", ctypes.c_uint32), ("log2_hashmap_size", ctypes.c_uint32),
                ("base_resolution", ctypes.c_uint32), ("log2_per_level_scale", ctypes.c_double), ("learning_rate", ctypes.c_float)]


class Split(ctypes.Structure):
    _fields_ = [("pixels", ctypes.c_void_p), ("camera", ctypes.c_void_p), ("frame_count", ctypes.c_uint32), ("width", ctypes.c_uint32),
                ("height", ctypes.c_uint32), ("focal_x", ctypes.c_float), ("focal_y", ctypes.c_float), ("principal_x", ctypes.c_float),
                ("principal_y", ctypes.c_float)]


class TrainStats(ctypes.Structure):
    _fields_ = [("step", ctypes.c_uint32), ("rays_per_batch", ctypes.c_uint32), ("measured_sample_count_before_compaction", ctypes.c_uint32),
                ("measured_sample_count", ctypes.c_uint32), ("density_grid_occupied_cells", ctypes.c_uint32), ("loss", ctypes.c_float),
                ("elapsed_ms", ctypes.c_float), ("density_grid_update_ms", ctypes.c_float), ("density_grid_occupancy_ratio", ctypes.c_float)]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


def trainer_config(n_levels=8, features_per_level=4, log2_hashmap_size=19, base_resolution=16, log2_per_level_scale=1.0,
                   learning_rate=1e-2) -> TrainerConfig:
    return TrainerConfig(n_levels, features_per_level, log2_hashmap_size, base_resolution, log2_per_level_scale, learning_rate)


def config0_trainer_config() -> TrainerConfig:
    return trainer_config(16, 2, 19, 16, math.log2(2048.0 / 16.0) / 15.0)


def config4_trainer_config() -> TrainerConfig:
    """the config-0 grid with log2 T = 22 (table beyond L2) and finest
    resolution 4096, b = exp(ln(4096/16)/15)."""
    return trainer_config(16, 2, 22, 16, math.log2(4096.0 / 16.0) / 15.0)


class InstantNGP:
    """Training / evaluation of one scene (ngp.train.ixx:40-53).  `dataset` is a dict with splits
    "train", "validation", "test", each a dict(pixels=uint8 [F][H][W][4], camera=float32 [F][12],
    focal=(fx, fy), principal=(cx, cy)) of host numpy arrays."""

    def __init__(self, dataset: dict, config: TrainerConfig | None = None) -> None:
        import numpy as np

        self._keep = []
        splits = []
        for name in ("train", "validation", "test"):
            d = dataset.get(name)
            if d is None or len(d["pixels"]) == 0:
                splits.append(None)
                continue
            px = np.ascontiguousarray(d["pixels"], np.uint8)
            cam = np.ascontiguousarray(d["camera"], np.float32)
            self._keep += [px, cam]
            f, h, w = px.shape[0], px.shape[1], px.shape[2]
            splits.append(Split(px.ctypes.data, cam.ctypes.data, f, w, h, d["focal"][0], d["focal"][1], d["principal"][0], d["principal"][1]))
        self.config = config if config is not None else trainer_config()
        self.handle = ctypes.c_void_p(0)
        ptrs = [ctypes.byref(s) if s is not None else None for s in splits]
        _check(lib().ngp_trainer_create(ctypes.byref(self.config), *ptrs, ctypes.byref(self.handle)), "ngp_trainer_create")
        self._keep = []
        self.test_size = None if splits[2] is None else (splits[2].width, splits[2].height)
        self.split_frames = {i: (0 if s is None else int(s.frame_count)) for i, s in enumerate(splits)}
        self.scene_scale = float(dataset.get("scene_scale", 0.33))
        self.step = 0

    def close(self) -> None:
        if self.handle:
            lib().ngp_trainer_destroy(self.handle)
            self.handle = ctypes.c_void_p(0)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def train(self, iters: int) -> dict:
        st = TrainStats()
        _check(lib().ngp_trainer_train(self.handle, ctypes.c_int32(iters), ctypes.byref(st)), "ngp_trainer_train")
        d = st.as_dict()
        self.step = int(d["step"])
        return d

    def layout(self) -> GridLayout:
        c = self.config
        return grid_layout(c.n_levels, c.features_per_level, c.log2_hashmap_size, c.base_resolution, c.log2_per_level_scale)

    def export_weights(self, path) -> None:
        """safetensors "instant-ngp-new.weights.v2" (InstantNGP::export_weights, ngp.train.cpp:231-296)."""
        import ngp_weights as weights

        weights.export_weights(path, self.get_params(), self.layout(), self.scene_scale)

    def load_weights(self, path) -> None:
        """Load a weights file before training (InstantNGP::load_weights, ngp.train.cpp:298-425);
        the optimizer state starts from zero, as in the reference."""
        import ngp_weights as weights

        if self.step != 0:
            raise RuntimeError("weights can only be loaded before training starts.")
        self.set_params(weights.load_weights(path, self.layout(), self.scene_scale))

    def write_test_images(self, output_dir="test") -> dict:
        """InstantNGP::test (ngp.train.cpp:183-229): test PSNR and one side-by-side comparison PNG
        per test image (target left, render right) as output_dir/test_NNNN.png."""
        from pathlib import Path

        from PIL import Image

        out = Path(output_dir)
        if out.exists() and not out.is_dir():
            raise RuntimeError(f"test output path '{out}' is not a directory.")
        out.mkdir(parents=True, exist_ok=True)
        res = self.test(with_images=True)
        for i, img in enumerate(res.pop("images")):
            Image.fromarray(img, "RGB").save(out / f"test_{i:04d}.png")
        res["output_dir"] = str(out)
        return res

    def _evaluate(self, split: int, begin: int, count: int, comparison=None):
        sse = ctypes.c_double(0.0)
        pixels = ctypes.c_uint64(0)
        cmp_ptr = None if comparison is None else ctypes.c_void_p(comparison.ctypes.data)
        _check(lib().ngp_trainer_evaluate(self.handle, ctypes.c_int(split), _u32(begin), _u32(count), cmp_ptr, ctypes.byref(sse),
                                          ctypes.byref(pixels)), "ngp_trainer_evaluate")
        return sse.value, pixels.value

    @staticmethod
    def _psnr(sse: float, pixels: int) -> tuple[float, float]:
        mse = sse / (pixels * 3.0)
        return mse, (float("inf") if mse <= 0 else -10.0 * math.log10(mse))

    def validate(self, count: int | None = None) -> dict:
        """Mean PSNR over the validation images (ngp.train.cpp:157-181)."""
        n = count if count is not None else self._count(1)
        sse, px = self._evaluate(1, 0, n)
        mse, psnr = self._psnr(sse, px)
        return {"image_count": n, "pixel_count": px, "mse": mse, "psnr": psnr}

    def test(self, count: int | None = None, with_images: bool = False) -> dict:
        """Test PSNR (ngp.train.cpp:183-229); optionally the side-by-side comparison images."""
        import numpy as np

        n = count if count is not None else self._count(2)
        sse_total, px_total, images = 0.0, 0, []
        for i in range(n):
            cmp = None
            if with_images:
                w, h = self.test_size
                cmp = np.zeros((h, 2 * w, 3), np.uint8)
            sse, px = self._evaluate(2, i, 1, cmp)
            sse_total += sse
            px_total += px
            if with_images:
                images.append(cmp)
        mse, psnr = self._psnr(sse_total, px_total)
        return {"image_count": n, "pixel_count": px_total, "mse": mse, "psnr": psnr, "images": images}

    def _count(self, split: int) -> int:
        return self.split_frames[split]

    def render(self, camera, width: int, height: int, focal, principal, out=None):
        import numpy as np
        import torch

        cam = np.ascontiguousarray(camera, np.float32)
        out = torch.empty((height * width, 3), dtype=torch.float32, device="cuda") if out is None else out
        _check(lib().ngp_trainer_render(self.handle, ctypes.c_void_p(cam.ctypes.data), _u32(width), _u32(height), _f32(focal[0]), _f32(focal[1]),
                                        _f32(principal[0]), _f32(principal[1]), _ptr(out)), "ngp_trainer_render")
        return out

    def render_tiles(self, camera, width: int, height: int, focal, principal, first_tile: int, tile_stride: int, out):
        """Render 64 x 64 tiles first_tile, first_tile + tile_stride, ... of the row-major tile grid
        into out [height * width][3] (other pixels untouched): rank r of N renders r, r + N, ..."""
        import numpy as np

        cam = np.ascontiguousarray(camera, np.float32)
        _check(lib().ngp_trainer_render_tiles(self.handle, ctypes.c_void_p(cam.ctypes.data), _u32(width), _u32(height), _f32(focal[0]),
                                              _f32(focal[1]), _f32(principal[0]), _f32(principal[1]), _u32(first_tile), _u32(tile_stride),
                                              _ptr(out)), "ngp_trainer_render_tiles")
        return out

    def set_segmented_eval(self, enabled: bool) -> None:
        """Segmented marching for evaluation and rendering (default) or the reference's
        march-everything-first flow; the images are identical."""
        _check(lib().ngp_trainer_set_segmented_eval(self.handle, ctypes.c_int(1 if enabled else 0)), "ngp_trainer_set_segmented_eval")

    def param_count(self) -> int:
        lib().ngp_trainer_param_count.restype = ctypes.c_uint32
        return int(lib().ngp_trainer_param_count(self.handle))

    def get_params(self):
        import numpy as np

        out = np.zeros(self.param_count(), np.float32)
        _check(lib().ngp_trainer_get_params(self.handle, ctypes.c_void_p(out.ctypes.data), _u32(out.size)), "ngp_trainer_get_params")
        return out

    def set_params(self, params) -> None:
        import numpy as np

        p = np.ascontiguousarray(params, np.float32)
        _check(lib().ngp_trainer_set_params(self.handle, ctypes.c_void_p(p.ctypes.data), _u32(p.size)), "ngp_trainer_set_params")

    PHASES = ("grid_update", "march", "inference_compact", "mlp_fwd_loss_pad", "mlp_bwd", "encode_bwd", "exchange", "adam")

    def set_run_ahead(self, enable: bool = True) -> None:
        """Run-ahead of the next step's grid-update first half when a train call returns (default
        on); off: a call's elapsed_ms covers exactly the work of its steps."""
        _check(lib().ngp_trainer_set_run_ahead(self.handle, ctypes.c_int(1 if enable else 0)), "ngp_trainer_set_run_ahead")

    def set_profiling(self, enable: bool = True) -> None:
        _check(lib().ngp_trainer_set_profiling(self.handle, ctypes.c_int(1 if enable else 0)), "ngp_trainer_set_profiling")

    def phase_times(self) -> dict:
        out = (ctypes.c_float * len(self.PHASES))()
        steps = ctypes.c_uint32(0)
        mean_n = ctypes.c_float(0)
        _check(lib().ngp_trainer_phase_times(self.handle, out, _u32(len(self.PHASES)), ctypes.byref(steps), ctypes.byref(mean_n)),
               "ngp_trainer_phase_times")
        return {"steps": steps.value, "mean_inference_samples": mean_n.value, "ms": dict(zip(self.PHASES, list(out)))}

    GRID_PHASES = ("grid_samples", "grid_encode", "grid_density", "grid_splat", "grid_ema_bitfield")

    def grid_phase_times(self) -> dict:
        """Per-kernel times of the profiled steps' grid updates (accumulated ms), the number of
        updates and their mean sample count."""
        out = (ctypes.c_float * len(self.GRID_PHASES))()
        updates = ctypes.c_uint32(0)
        mean_n = ctypes.c_float(0)
        _check(lib().ngp_trainer_grid_phase_times(self.handle, out, _u32(len(self.GRID_PHASES)), ctypes.byref(updates), ctypes.byref(mean_n)),
               "ngp_trainer_grid_phase_times")
        return {"updates": updates.value, "mean_samples": mean_n.value, "ms": dict(zip(self.GRID_PHASES, list(out)))}

    def join(self, unique_id: bytes, world: int, rank: int) -> None:
        """Join a data-parallel group of `world` trainers (one per GPU) before the first step."""
        buf = (ctypes.c_uint8 * 128).from_buffer_copy(unique_id[:128].ljust(128, b"\0"))
        _check(lib().ngp_trainer_join(self.handle, buf, ctypes.c_int(world), ctypes.c_int(rank)), "ngp_trainer_join")

    def train_guarded(self, iters: int, health: RankHealth) -> dict:
        """train(1) `iters` times, each after health.before_step: a rank that left (or stopped) is
        reported on the host before this rank launches the step's collectives."""
        st = {}
        for _ in range(iters):
            health.before_step(self.step)
            st = self.train(1)
        return st

    LOSSES = {"l2": 0, "huber": 1}

    def set_loss(self, kind: str) -> None:
        """Training loss: "l2" (the reference's, default) or "huber" (delta 0.1, scaled by 1/5)."""
        _check(lib().ngp_trainer_set_loss(self.handle, ctypes.c_int(self.LOSSES[kind])), "ngp_trainer_set_loss")

    def exchange_mode(self) -> str:
        """The joined trainer's gradient exchange: "none", "nccl" or "peer" (one fused kernel
        over NVLink peer memory)."""
        return {0: "none", 1: "nccl", 2: "peer"}[int(lib().ngp_trainer_exchange_mode(self.handle))]

    def set_collective_timeout(self, ms: float) -> None:
        """Collectives (and waits for the stream that runs them) that take longer abort the
        communicator and raise (NGP_ERR_TIMEOUT)."""
        _check(lib().ngp_trainer_set_collective_timeout(self.handle, ctypes.c_double(ms)), "ngp_trainer_set_collective_timeout")

    def join_process_group(self) -> None:
        """Join using the current torch.distributed process group to share the NCCL id."""
        import torch.distributed as dist

        world, rank = dist.get_world_size(), dist.get_rank()
        if world == 1:
            return
        self.join(share_nccl_id(), world, rank)

    def get_grid(self):
        import numpy as np

        bits = np.zeros(GRID_CELLS // 8, np.uint8)
        vals = np.zeros(GRID_CELLS, np.float32)
        _check(lib().ngp_trainer_get_grid(self.handle, ctypes.c_void_p(bits.ctypes.data), ctypes.c_void_p(vals.ctypes.data)), "ngp_trainer_get_grid")
        return bits, vals


class RankHealth:
    """Host-side liveness of the ranks of a data-parallel job, kept in a torch.distributed store (no
    GPU involved; no counterpart in the single-GPU reference).

    Before a step that runs collectives, each rank calls before_step(step): it publishes the step
    and waits until every other rank has published that step or a later one.  A rank that leaves
    the job calls leave() between steps; the others raise RuntimeError naming it at their next
    before_step.  A rank that stops without leaving is reported once `timeout_s` expires.  Either
    way the remaining ranks learn of it on the host, before they launch a collective that could
    not complete (the trainer's collective timeout is the second line of defence)."""

    def __init__(self, store=None, world: int | None = None, rank: int | None = None, timeout_s: float = 30.0, prefix: str = "ngp_health"):
        import torch.distributed as dist

        self.store = store if store is not None else dist.distributed_c10d._get_default_store()
        self.world = dist.get_world_size() if world is None else world
        self.rank = dist.get_rank() if rank is None else rank
        self.timeout_s = timeout_s
        self.prefix = prefix

    def _key(self, kind: str, rank: int) -> str:
        return f"{self.prefix}/{kind}/{rank}"

    def before_step(self, step: int) -> None:
        import time

        self.store.set(self._key("step", self.rank), str(step))
        pending = [r for r in range(self.world) if r != self.rank]
        deadline = time.monotonic() + self.timeout_s
        while pending:
            for r in list(pending):
                if self.store.check([self._key("left", r)]):
                    raise RuntimeError(f"rank {r} left the data-parallel job before step {step}")
                if self.store.check([self._key("step", r)]) and int(self.store.get(self._key("step", r))) >= step:
                    pending.remove(r)
            if pending and time.monotonic() > deadline:
                raise RuntimeError(f"ranks {pending} did not reach step {step} within {self.timeout_s} s")
            if pending:
                time.sleep(0.001)

    def leave(self) -> None:
        self.store.set(self._key("left", self.rank), "1")


def share_nccl_id() -> bytes:
    """Rank 0 creates an NCCL unique id and broadcasts it over the current torch.distributed group
    (any backend: the id travels in a CPU tensor for gloo, a device tensor for nccl)."""
    import torch
    import torch.distributed as dist

    rank = dist.get_rank()
    uid = nccl_unique_id() if rank == 0 else bytes(128)
    device = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor(list(uid), dtype=torch.uint8, device=device)
    dist.broadcast(t, src=0)
    return bytes(t.cpu().tolist())


FAULT_SITES = {"alloc": 1, "launch": 2, "collective": 3}


def fault_inject(site: str, countdown: int) -> None:
    """Arm host-side fault injection: the countdown-th allocation / kernel launch / collective of
    the library from now fails with an "injected fault" error (0 disarms).  No GPU fault is raised."""
    _check(lib().ngp_fault_inject(ctypes.c_int(FAULT_SITES[site]), ctypes.c_int64(countdown)), "ngp_fault_inject")


def nccl_unique_id() -> bytes:
    buf = (ctypes.c_uint8 * 128)()
    _check(lib().ngp_nccl_unique_id(buf, ctypes.c_size_t(128)), "ngp_nccl_unique_id")
    return bytes(buf)
