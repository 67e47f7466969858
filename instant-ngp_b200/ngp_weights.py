"""Weights checkpoint: the reference's safetensors format "instant-ngp-new.weights.v2"
(InstantNGP::export_weights / load_weights, ngp.train.cpp:231-425), byte-compatible.

Layout: an 8-byte little-endian header length, the header as compact JSON with sorted keys (the
reference serialises an nlohmann::json object, whose keys are ordered), then the fp32 tensors in
the order density_mlp.input, density_mlp.output, rgb_mlp.input, rgb_mlp.hidden, rgb_mlp.output,
hash_grid.params, each [out][in] (the grid [entries][features]), back to back.  The metadata
records the grid and network shape as strings and the scene scale as "%.9g"; loading requires
the metadata to match the model exactly and every value to be finite, as the reference does.
"""
from __future__ import annotations

import json
import math
import struct
from pathlib import Path

import numpy as np

FORMAT = "instant-ngp-new.weights.v2"
MLP_WIDTH = 64
DENSITY_OUTPUT_WIDTH = 16
DIRECTION_OUTPUT_WIDTH = 16
NETWORK_OUTPUT_WIDTH = 16
MAX_HEADER = 100 * 1024 * 1024


def _tensors(grid_entries: int, features: int, grid_width: int):
    """(name, parameter offset, rows, cols) in file order (ngp.train.cpp:244-251)."""
    rgb_in = DENSITY_OUTPUT_WIDTH + DIRECTION_OUTPUT_WIDTH
    d_in = 0
    d_out = d_in + MLP_WIDTH * grid_width
    r_in = d_out + DENSITY_OUTPUT_WIDTH * MLP_WIDTH
    r_hid = r_in + MLP_WIDTH * rgb_in
    r_out = r_hid + MLP_WIDTH * MLP_WIDTH
    grid = r_out + NETWORK_OUTPUT_WIDTH * MLP_WIDTH
    return [("density_mlp.input.weight", d_in, MLP_WIDTH, grid_width), ("density_mlp.output.weight", d_out, DENSITY_OUTPUT_WIDTH, MLP_WIDTH),
            ("rgb_mlp.input.weight", r_in, MLP_WIDTH, rgb_in), ("rgb_mlp.hidden.weight", r_hid, MLP_WIDTH, MLP_WIDTH),
            ("rgb_mlp.output.weight", r_out, NETWORK_OUTPUT_WIDTH, MLP_WIDTH), ("hash_grid.params", grid, grid_entries, features)]


def metadata(layout, scene_scale: float) -> dict:
    """The "__metadata__" object (ngp.train.cpp:262-278)."""
    L, F = int(layout.n_levels), int(layout.features_per_level)
    return {"format": FORMAT, "grid_n_levels": str(L), "grid_features_per_level": str(F), "grid_base_resolution": str(int(layout.base_resolution)),
            "grid_log2_hashmap_size": str(int(layout.log2_hashmap_size)), "mlp_width": str(MLP_WIDTH), "density_hidden_layers": "1",
            "rgb_hidden_layers": "2", "density_output_width": str(DENSITY_OUTPUT_WIDTH), "direction_output_width": str(DIRECTION_OUTPUT_WIDTH),
            "rgb_input_width": str(DENSITY_OUTPUT_WIDTH + DIRECTION_OUTPUT_WIDTH), "network_output_width": str(NETWORK_OUTPUT_WIDTH),
            "grid_offsets": ",".join(str(int(layout.offsets[i])) for i in range(L + 1)),
            "scene_scale": format(float(np.float32(scene_scale)), ".9g")}


def _header(layout, scene_scale: float) -> tuple[str, list]:
    L, F = int(layout.n_levels), int(layout.features_per_level)
    tensors = _tensors(int(layout.offsets[L]), F, L * F)
    header = {"__metadata__": metadata(layout, scene_scale)}
    off = 0
    for name, _, rows, cols in tensors:
        n = rows * cols * 4
        header[name] = {"dtype": "F32", "shape": [rows, cols], "data_offsets": [off, off + n]}
        off += n
    return json.dumps(header, sort_keys=True, separators=(",", ":")), tensors


def export_weights(path, params: np.ndarray, layout, scene_scale: float) -> None:
    """Write the fp32 parameters [MLP | grid] (the trainer's packing) to `path`."""
    path = Path(path)
    if str(path) == "":
        raise RuntimeError("weights export path must not be empty.")
    if path.parent != Path("") and not path.parent.is_dir():
        raise RuntimeError(f"weights export parent directory '{path.parent}' does not exist.")
    params = np.ascontiguousarray(params, dtype="<f4")
    text, tensors = _header(layout, scene_scale)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(text)))
        f.write(text.encode())
        for _, off, rows, cols in tensors:
            f.write(params[off:off + rows * cols].tobytes())


def load_weights(path, layout, scene_scale: float) -> np.ndarray:
    """Read and validate a weights file against the model's shape; returns the fp32 parameters."""
    path = Path(path)
    if not path.is_file():
        raise RuntimeError(f"weights file '{path}' does not exist.")
    raw = path.read_bytes()
    if len(raw) < 8:
        raise RuntimeError("weights file is too small for a safetensors header.")
    (hlen,) = struct.unpack("<Q", raw[:8])
    if hlen == 0 or hlen > MAX_HEADER:
        raise RuntimeError("invalid safetensors header length.")
    if 8 + hlen > len(raw):
        raise RuntimeError("safetensors header length exceeds file size.")
    text = raw[8:8 + hlen].decode()
    if not text.startswith("{"):
        raise RuntimeError("safetensors header must begin with '{'.")
    header = json.loads(text)
    if not isinstance(header, dict):
        raise RuntimeError("safetensors header must be a JSON object.")
    _, tensors = _header(layout, scene_scale)
    if len(header) != len(tensors) + 1:
        raise RuntimeError("safetensors header contains unexpected tensors.")
    if header.get("__metadata__") != metadata(layout, scene_scale):
        raise RuntimeError("safetensors metadata does not match the current InstantNGP configuration.")
    total = tensors[-1][1] + tensors[-1][2] * tensors[-1][3]
    params = np.zeros(total, np.float32)
    data = memoryview(raw)[8 + hlen:]
    expected = 0
    for name, off, rows, cols in tensors:
        t = header.get(name)
        if not isinstance(t, dict) or len(t) != 3:
            raise RuntimeError(f"safetensors tensor '{name}' has an invalid header.")
        if t.get("dtype") != "F32":
            raise RuntimeError(f"safetensors tensor '{name}' must use dtype F32.")
        if t.get("shape") != [rows, cols]:
            raise RuntimeError(f"safetensors tensor '{name}' shape mismatch.")
        n = rows * cols * 4
        if t.get("data_offsets") != [expected, expected + n]:
            raise RuntimeError(f"safetensors tensor '{name}' data_offsets mismatch.")
        expected += n
    if expected != len(data):
        raise RuntimeError("safetensors data buffer size does not match tensor offsets.")
    pos = 0
    for _, off, rows, cols in tensors:
        params[off:off + rows * cols] = np.frombuffer(data[pos:pos + rows * cols * 4], dtype="<f4")
        pos += rows * cols * 4
    if not np.isfinite(params).all():
        raise RuntimeError("weights file contains non-finite values.")
    return params
