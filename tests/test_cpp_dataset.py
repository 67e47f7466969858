"""The C++23 scene loaders (include/ngp_b200_dataset.hpp) against the Python loaders, which
tests/test_io.py checks against an independent float32 evaluation of the reference's camera
conversion: the same frames, pixels, cameras (bit for bit) and intrinsics, for NeRF-synthetic and
DD-NeRF fixtures; the PNG decoder against Pillow on every 8-bit colour type, filter choice and
compression level; the reference's error messages on bad inputs.  No GPU needed."""
from __future__ import annotations

import ctypes
import json
import shutil
import subprocess

import numpy as np
import pytest
from test_io import _c2w, make_nerf_synthetic

import ngp_dataset as datasets
from conftest import ROOT


@pytest.fixture(scope="module")
def probe(tmp_path_factory, ngp):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    out = tmp_path_factory.mktemp("cppds") / "libcpp_dataset_probe.so"
    lib_dir = ROOT / "instant-ngp_b200"
    cmd = [gxx, "-std=c++23", "-O1", "-Wall", "-Wextra", "-Werror", "-shared", "-fPIC", f"-I{ROOT / 'include'}",
           str(ROOT / "tests/cpp/cpp_dataset_probe.cpp"), f"-L{lib_dir}", "-lngp_b200", f"-Wl,-rpath,{lib_dir}", "-o", str(out)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    return ctypes.CDLL(str(out))


def _load(probe, path, kind, scale):
    err = ctypes.create_string_buffer(1024)
    counts, dims = np.zeros(3, np.uint32), np.zeros(6, np.uint32)
    P = lambda a: ctypes.c_void_p(a.ctypes.data)  # noqa: E731
    rc = probe.probe_dataset_shape(str(path).encode(), kind, ctypes.c_float(scale), P(counts), P(dims), err, ctypes.c_size_t(1024))
    if rc != 0:
        raise RuntimeError(err.value.decode())
    out = {}
    for s, name in enumerate(("train", "validation", "test")):
        n, w, h = int(counts[s]), int(dims[2 * s]), int(dims[2 * s + 1])
        px, cam, intr = np.zeros((n, h, w, 4), np.uint8), np.zeros((n, 12), np.float32), np.zeros((n, 4), np.float32)
        assert probe.probe_dataset_split(str(path).encode(), kind, ctypes.c_float(scale), s, P(px), P(cam), P(intr), err, ctypes.c_size_t(1024)) == 0
        out[name] = (px, cam, intr)
    return out


def _same(cpp, py):
    for name in ("train", "validation", "test"):
        px, cam, intr = cpp[name]
        d = py[name]
        assert px.shape == d["pixels"].shape and (px == d["pixels"]).all()
        assert cam.tobytes() == np.ascontiguousarray(d["camera"], np.float32).tobytes()
        for row in intr:
            assert (float(row[0]), float(row[1])) == d["focal"] and (float(row[2]), float(row[3])) == d["principal"]


def test_nerf_synthetic_same_as_python(probe, tmp_path):
    make_nerf_synthetic(tmp_path, n=(4, 2, 3), w=17, h=9, seed=5)
    _same(_load(probe, tmp_path, 0, 0.33), datasets.load_nerf_synthetic(tmp_path, 0.33))


def test_dd_nerf_same_as_python(probe, tmp_path):
    from PIL import Image

    rng = np.random.default_rng(2)
    frames = []
    (tmp_path / "images").mkdir()
    for i in range(30):
        name = f"frame_{i:03d}.png"
        Image.fromarray(rng.integers(0, 256, (7, 9, 4), dtype=np.uint8), "RGBA").save(tmp_path / "images" / name)
        frames.append({"file_path": f"images/{name}", "transform_matrix": _c2w(rng)})
    text = json.dumps({"w": 9, "h": 7, "fl_x": 8.5, "fl_y": 8.25, "cx": 4.5, "cy": 3.5, "frames": frames}, indent=1)
    (tmp_path / "cameras.json").write_text("// written by the test\n" + text)  # comments are allowed, as in the reference
    _same(_load(probe, tmp_path, 1, 0.5), _python_dd(tmp_path, text, 0.5))


def _python_dd(tmp_path, text, scale):
    # the Python loader reads strict JSON: give it the same file without the comment line
    alt = tmp_path.parent / (tmp_path.name + "_strict")
    shutil.copytree(tmp_path, alt)
    (alt / "cameras.json").write_text(text)
    return datasets.load_dd_nerf(alt, scale)


@pytest.mark.parametrize("mode", ["RGBA", "RGB", "L", "LA", "P", "P_trns", "L_trns", "RGB_trns"])
@pytest.mark.parametrize("level", [0, 1, 6, 9])
def test_png_decoder_matches_pillow(probe, tmp_path, mode, level):
    from PIL import Image

    rng = np.random.default_rng(len(mode) * 10 + level)
    h, w = 23, 31
    smooth = (np.add.outer(np.arange(h), np.arange(w)) * 3 % 256).astype(np.uint8)  # filters other than None pay off here
    noise = rng.integers(0, 256, (h, w), dtype=np.uint8)
    base = np.where(rng.random((h, w)) < 0.5, smooth, noise)
    info = {}
    if mode in ("RGBA", "RGB"):
        img = Image.fromarray(np.stack([base, noise, smooth, noise[::-1]][: len(mode)], -1), mode)
    elif mode in ("L", "LA"):
        img = Image.fromarray(base if mode == "L" else np.stack([base, noise], -1), mode)
    elif mode.startswith("P"):
        img = Image.fromarray(base % 64, "P")
        img.putpalette(list(rng.integers(0, 256, 64 * 3)))
        if mode == "P_trns":
            info["transparency"] = bytes(rng.integers(0, 256, 40).tolist())
    elif mode == "L_trns":
        img, info["transparency"] = Image.fromarray(base, "L"), int(base[3, 4])
    else:
        img, info["transparency"] = Image.fromarray(np.stack([base, base, base], -1), "RGB"), (int(base[1, 1]),) * 3
    path = tmp_path / "x.png"
    img.save(path, compress_level=level, **info)
    want = np.asarray(Image.open(path).convert("RGBA"))
    got, wh, err = np.zeros(h * w * 4, np.uint8), np.zeros(2, np.uint32), ctypes.create_string_buffer(1024)
    rc = probe.probe_png(str(path).encode(), ctypes.c_void_p(got.ctypes.data), ctypes.c_size_t(got.size), ctypes.c_void_p(wh.ctypes.data), err,
                         ctypes.c_size_t(1024))
    assert rc == 0, err.value
    assert tuple(wh) == (w, h)
    assert (got.reshape(h, w, 4) == want).all()


def test_reference_error_messages(probe, tmp_path):
    with pytest.raises(RuntimeError, match="scene scale must be finite and positive"):
        _load(probe, tmp_path, 0, -1.0)
    with pytest.raises(RuntimeError, match="missing cameras.json"):
        _load(probe, tmp_path, 1, 0.33)
    (tmp_path / "cameras.json").write_text('{"w": 4, "h": 4, "fl_x": 1, "fl_y": 1, "cx": 9, "cy": 1, "frames": [{}]}')
    (tmp_path / "images").mkdir()
    with pytest.raises(RuntimeError, match="invalid principal point"):
        _load(probe, tmp_path, 1, 0.33)
