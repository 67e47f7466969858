"""Scene loaders, the weights checkpoint format and the command line (the reference's
ngp.dataset.cpp, InstantNGP::export_weights / load_weights and main.cpp) on the CPU.

The NeRF-synthetic and DD-NeRF fixtures are written here (small PNGs and JSON), since the
reference ships no data.  Cameras are checked against an independent float32 evaluation of the
conversion (ngp.dataset.cpp:47-65); the FNV-1a split hash against the published FNV test vectors;
the weights file byte for byte against a header and payload assembled here from the format
description.  The GPU tier runs the command line end to end (tests/test_io_gpu.py)."""
from __future__ import annotations

import json
import math
import struct
from pathlib import Path

import numpy as np
import pytest

import cli
import ngp_dataset as datasets
import ngp_weights as weights


def _write_png(path: Path, rgba: np.ndarray) -> None:
    from PIL import Image

    path.parent.mkdir(parents=True, exist_ok=True)
    Image.fromarray(rgba, "RGBA").save(path)


def _c2w(rng) -> list:
    m = np.eye(4)
    q, _ = np.linalg.qr(rng.normal(size=(3, 3)))
    m[:3, :3] = q
    m[:3, 3] = rng.uniform(-4, 4, 3)
    return m.tolist()


def make_nerf_synthetic(root: Path, n=(3, 2, 2), w=12, h=10, seed=0) -> dict:
    rng = np.random.default_rng(seed)
    out = {}
    for split, count in zip(("train", "val", "test"), n):
        frames, imgs = [], []
        for i in range(count):
            img = rng.integers(0, 256, (h, w, 4), dtype=np.uint8)
            _write_png(root / split / f"r_{i}.png", img)
            mat = _c2w(rng)
            frames.append({"file_path": f"./{split}/r_{i}", "transform_matrix": mat})
            imgs.append((img, mat))
        (root / f"transforms_{split}.json").write_text(json.dumps({"camera_angle_x": 0.6911112070083618, "frames": frames}))
        out[split] = imgs
    return out


def expected_camera(mat, scale) -> np.ndarray:
    """The conversion written out element by element in float32."""
    m = np.array(mat, np.float32)
    f = np.float32
    pos = [f(f(m[r, 3] * f(scale)) + f(0.5)) for r in range(3)]
    # columns: x = m[:,0], y = -m[:,1], z = -m[:,2]; axes permuted (x, y, z) -> (y, z, x)
    x, y, z = m[:3, 0], -m[:3, 1], -m[:3, 2]
    return np.array([x[1], x[2], x[0], y[1], y[2], y[0], z[1], z[2], z[0], pos[1], pos[2], pos[0]], np.float32)


def test_nerf_synthetic_loader(tmp_path):
    truth = make_nerf_synthetic(tmp_path)
    ds = datasets.load_nerf_synthetic(tmp_path, 0.33)
    for split, key in (("train", "train"), ("val", "validation"), ("test", "test")):
        d = ds[key]
        assert d["pixels"].shape == (len(truth[split]), 10, 12, 4)
        for i, (img, mat) in enumerate(truth[split]):
            assert (d["pixels"][i] == img).all()
            assert d["camera"][i].tobytes() == expected_camera(mat, 0.33).tobytes()
        focal = np.float32(np.float32(0.5) * np.float32(12)) / np.float32(math.tan(float(np.float32(0.6911112070083618) * np.float32(0.5))))
        assert d["focal"] == (float(focal), float(focal)) and d["principal"] == (6.0, 5.0)
    assert ds["scene_scale"] == float(np.float32(0.33))
    fmt = datasets.load_dataset(tmp_path)[1]
    assert fmt == "nerf-synthetic"


def test_camera_conversion_matches_scene_generator():
    """The loader's conversion and the one the procedural scenes use agree (ngp.dataset.cpp:47-65)."""
    import workloads

    rng = np.random.default_rng(3)
    for _ in range(5):
        c2w = np.array(_c2w(rng), np.float32)
        a = datasets.ngp_camera(c2w, 0.33)
        b = workloads.nerf_to_ngp_camera(c2w.astype(np.float64), 0.33)
        np.testing.assert_allclose(a, b, rtol=0, atol=2e-7)


def test_fnv1a_vectors():
    # published FNV-1a 64-bit test vectors
    assert datasets.fnv1a64("") == 0xCBF29CE484222325
    assert datasets.fnv1a64("a") == 0xAF63DC4C8601EC8C
    assert datasets.fnv1a64("foobar") == 0x85944171F73967E8


def test_dd_nerf_loader_split(tmp_path):
    rng = np.random.default_rng(1)
    frames, truth = [], {}
    names = [f"img_{i:03d}.png" for i in range(40)]
    for name in names:
        img = rng.integers(0, 256, (6, 8, 4), dtype=np.uint8)
        _write_png(tmp_path / "images" / name, img)
        mat = _c2w(rng)
        frames.append({"file_path": f"images/{name}", "transform_matrix": mat})
        truth[name] = (img, mat)
    (tmp_path / "cameras.json").write_text(json.dumps({"w": 8, "h": 6, "fl_x": 7.5, "fl_y": 7.25, "cx": 4.0, "cy": 3.0, "frames": frames}))
    ds = datasets.load_dd_nerf(tmp_path, 0.5)
    buckets = {"train": [], "validation": [], "test": []}
    for name in names:
        k = datasets.fnv1a64(name) % 10
        buckets["test" if k == 0 else "validation" if k == 1 else "train"].append(name)
    for split, members in buckets.items():
        d = ds[split]
        assert len(d["pixels"]) == len(members) > 0
        for i, name in enumerate(members):
            assert (d["pixels"][i] == truth[name][0]).all()
            assert d["camera"][i].tobytes() == expected_camera(truth[name][1], 0.5).tobytes()
        assert d["focal"] == (7.5, 7.25) and d["principal"] == (4.0, 3.0)
    assert datasets.load_dataset(tmp_path)[1] == "dd-nerf-dataset"


def test_loader_errors(tmp_path):
    with pytest.raises(RuntimeError):
        datasets.load_nerf_synthetic(tmp_path, -1.0)
    with pytest.raises(RuntimeError):
        datasets.load_dd_nerf(tmp_path)  # no cameras.json
    with pytest.raises(RuntimeError):
        datasets.load_dataset(tmp_path)  # no marker set


class _Layout:
    """Stand-in for ngp_grid_layout (the reference's compiled 8 x 4 grid: offsets of
    ngp.train.h:44-56 for base resolution 16 doubling per level, T = 2^19)."""

    def __init__(self):
        self.n_levels, self.features_per_level, self.base_resolution, self.log2_hashmap_size = 8, 4, 16, 19
        offs, cur = [], 0
        for lvl in range(8):
            r = 16 << lvl
            pos = min((min(r ** 3, 0xFFFFFFFF // 2) + 7) // 8 * 8, 1 << 19)
            offs.append(cur)
            cur += pos
        self.offsets = offs + [cur]


def test_weights_file_bytes_and_roundtrip(tmp_path):
    lay = _Layout()
    n = 10240 + lay.offsets[8] * 4
    assert n == 11692032  # the reference's total parameter count
    params = np.random.default_rng(0).standard_normal(n).astype(np.float32)
    path = tmp_path / "w.safetensors"
    weights.export_weights(path, params, lay, 0.33)
    raw = path.read_bytes()
    # assemble the expected file independently
    meta = {"density_hidden_layers": "1", "density_output_width": "16", "direction_output_width": "16", "format": "instant-ngp-new.weights.v2",
            "grid_base_resolution": "16", "grid_features_per_level": "4", "grid_log2_hashmap_size": "19", "grid_n_levels": "8",
            "grid_offsets": ",".join(map(str, lay.offsets)), "mlp_width": "64", "network_output_width": "16", "rgb_hidden_layers": "2",
            "rgb_input_width": "32", "scene_scale": "0.330000013"}
    order = [("density_mlp.input.weight", 0, 64, 32), ("density_mlp.output.weight", 2048, 16, 64), ("rgb_mlp.input.weight", 3072, 64, 32),
             ("rgb_mlp.hidden.weight", 5120, 64, 64), ("rgb_mlp.output.weight", 9216, 16, 64), ("hash_grid.params", 10240, lay.offsets[8], 4)]
    off, offs = 0, {}
    for name, _, r, c in order:
        offs[name] = (off, off + r * c * 4)
        off += r * c * 4
    header = '{"__metadata__":{' + ",".join(f'"{k}":"{v}"' for k, v in sorted(meta.items())) + "}"
    for name, _, r, c in sorted(order):
        header += f',"{name}":{{"data_offsets":[{offs[name][0]},{offs[name][1]}],"dtype":"F32","shape":[{r},{c}]}}'
    header += "}"
    payload = b"".join(params[o:o + r * c].tobytes() for _, o, r, c in order)
    assert raw == struct.pack("<Q", len(header)) + header.encode() + payload
    back = weights.load_weights(path, lay, 0.33)
    assert back.tobytes() == params.tobytes()


def test_weights_validation_errors(tmp_path):
    lay = _Layout()
    n = 10240 + lay.offsets[8] * 4
    params = np.zeros(n, np.float32)
    path = tmp_path / "w.safetensors"
    weights.export_weights(path, params, lay, 0.33)
    with pytest.raises(RuntimeError, match="metadata"):
        weights.load_weights(path, lay, 0.5)  # another scene scale
    raw = bytearray(path.read_bytes())
    raw[-4:] = np.array([np.nan], np.float32).tobytes()
    bad = tmp_path / "nan.safetensors"
    bad.write_bytes(bytes(raw))
    with pytest.raises(RuntimeError, match="non-finite"):
        weights.load_weights(bad, lay, 0.33)
    short = tmp_path / "short.safetensors"
    short.write_bytes(path.read_bytes()[:-4])
    with pytest.raises(RuntimeError, match="data buffer size"):
        weights.load_weights(short, lay, 0.33)
    with pytest.raises(RuntimeError, match="does not exist"):
        weights.load_weights(tmp_path / "missing", lay, 0.33)


def test_cli_argument_errors(tmp_path, capsys):
    assert cli.main([str(tmp_path / "nope")]) == 2
    make_nerf_synthetic(tmp_path)
    (tmp_path / "cameras.json").write_text("{}")
    (tmp_path / "images").mkdir()
    assert cli.main([str(tmp_path)]) == 2  # both marker sets
    assert "exactly one supported dataset marker set" in capsys.readouterr().out
    with pytest.raises(SystemExit):
        cli.main(["--steps", "0", str(tmp_path)])
    with pytest.raises(SystemExit):
        cli.main([str(tmp_path), "--dataset", str(tmp_path)])


# ---- scene-scale sweep (benchmark.cpp) ----------------------------------------------------------
import scale_sweep


def test_sweep_coarse_parsing():
    assert scale_sweep.parse_coarse("0.5,0.25,1") == [0.25, 0.5, 1.0]
    for bad in ("1", "0.5,-1", "0.5,,1", "0.5,0.5000001", "a,1"):
        with pytest.raises(ValueError):
            scale_sweep.parse_coarse(bad)


def test_sweep_refine_candidates():
    coarse = scale_sweep.parse_coarse(scale_sweep.DEFAULT_COARSE)
    # interior best: between its neighbours, log-spaced, the best in the middle
    c = scale_sweep.refine_candidates(coarse, 0.5, 5)
    lo, hi = 0.3535534, 0.7071068
    want = [math.exp(math.log(lo) * (1 - t) + math.log(0.5) * t) for t in (0.0, 0.5)] + [0.5] + \
           [math.exp(math.log(0.5) * (1 - t) + math.log(hi) * t) for t in (0.5, 1.0)]
    np.testing.assert_allclose(c, want, rtol=1e-12)
    # edge best: the missing neighbour is extrapolated by the neighbouring ratio
    c0 = scale_sweep.refine_candidates(coarse, 0.125, 3)
    np.testing.assert_allclose([c0[0], c0[1], c0[2]], [0.125 / (0.1767767 / 0.125), 0.125, 0.1767767], rtol=1e-12)
    cn = scale_sweep.refine_candidates(coarse, 4.0, 3)
    np.testing.assert_allclose([cn[0], cn[2]], [2.8284271, 4.0 * (4.0 / 2.8284271)], rtol=1e-12)


def test_sweep_best_and_csv():
    rows = [{"stage": "coarse", "failed": False, "final_psnr": 30.0, "scene_scale": 0.5},
            {"stage": "coarse", "failed": False, "final_psnr": 30.04, "scene_scale": 0.25},   # within 0.05 dB, smaller: wins
            {"stage": "coarse", "failed": True, "final_psnr": 40.0, "scene_scale": 1.0},
            {"stage": "refine", "failed": False, "final_psnr": 99.0, "scene_scale": 2.0}]
    assert scale_sweep.best_index(rows, "coarse") == 1
    r = {"stage": "coarse", "rank": 3, "scene_scale": 0.35355338, "failed": True, "error": 'bad "x"', "final_step": 10, "best_validation_step": 5,
         "final_psnr": 21.123456789, "final_mse": 0.0077, "best_psnr": 22.0, "best_mse": 0.006, "final_loss": 0.01, "occupancy_ratio": 0.25,
         "occupied_cells": 524288, "average_samples": 1000, "average_compacted": 500, "train_ms": 1234.5, "validation_ms": 12.0,
         "steps_per_second": 8.1}
    assert scale_sweep.csv_row(r) == 'coarse,3,0.353553,failed,"bad ""x""",10,5,21.1235,0.0077,22,0.006,0.01,0.25,524288,1000,500,1234.5,12,8.1'
    assert scale_sweep.CSV_HEADER.split(",")[0:4] == ["stage", "rank", "scene_scale", "status"]


def test_sweep_argument_errors(tmp_path):
    assert scale_sweep.main(["--dataset", str(tmp_path / "none")]) == 2
    assert scale_sweep.main(["--dataset", str(tmp_path), "--refine-count", "4"]) == 2
    assert scale_sweep.main(["--dataset", str(tmp_path), "--coarse-scales", "1"]) == 2
    assert scale_sweep.main(["--dataset", str(tmp_path)]) == 2  # no marker set
