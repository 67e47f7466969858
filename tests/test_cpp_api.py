"""The C++23 host interface (include/ngp_b200_train.hpp): compiles with g++ -std=c++23 against the
library; its weights file is byte-identical to the Python writer's (which matches the reference
format byte for byte, tests/test_io.py), reads back, and rejects a mismatching model; its PNG
decodes to the given pixels.  On a GPU, one InstantNGP lifecycle runs through it."""
from __future__ import annotations

import ctypes
import math
import shutil
import struct
import subprocess
import zlib

import numpy as np
import pytest

from conftest import ROOT

import ngp_weights
import workloads


@pytest.fixture(scope="module")
def probe(tmp_path_factory, ngp):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    out = tmp_path_factory.mktemp("cpp") / "libcpp_api_probe.so"
    lib_dir = ROOT / "instant-ngp_b200"
    cmd = [gxx, "-std=c++23", "-O1", "-Wall", "-Wextra", "-Werror", "-shared", "-fPIC", f"-I{ROOT / 'include'}", str(ROOT / "tests/cpp/cpp_api_probe.cpp"),
           f"-L{lib_dir}", "-lngp_b200", f"-Wl,-rpath,{lib_dir}", "-o", str(out)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    return ctypes.CDLL(str(out))


def _err():
    return ctypes.create_string_buffer(1024)


LAYOUT = (16, 2, 19, 16, math.log2(128.0) / 15.0)


def _layout_args():
    L, F, T, B, s = LAYOUT
    return [ctypes.c_uint32(L), ctypes.c_uint32(F), ctypes.c_uint32(T), ctypes.c_uint32(B), ctypes.c_double(s)]


def test_header_equals_python_writer(probe, ngp):
    buf, err = ctypes.create_string_buffer(8192), _err()
    assert probe.probe_header(*_layout_args(), ctypes.c_float(0.33), buf, ctypes.c_size_t(8192), err, ctypes.c_size_t(1024)) == 0, err.value
    text, _ = ngp_weights._header(ngp.grid_layout(*LAYOUT), 0.33)
    assert buf.value.decode() == text


def test_weights_bytes_match_python_and_round_trip(probe, ngp, tmp_path):
    layout = ngp.grid_layout(*LAYOUT)
    n = 10240 + int(layout.n_params)
    params = np.random.default_rng(3).uniform(-1, 1, n).astype(np.float32)
    err = _err()
    cpp_file, py_file = tmp_path / "cpp.safetensors", tmp_path / "py.safetensors"
    rc = probe.probe_write_weights(str(cpp_file).encode(), ctypes.c_void_p(params.ctypes.data), *_layout_args(), ctypes.c_float(0.33), err,
                                   ctypes.c_size_t(1024))
    assert rc == 0, err.value
    ngp_weights.export_weights(py_file, params, layout, 0.33)
    assert cpp_file.read_bytes() == py_file.read_bytes()
    back = np.zeros(n, np.float32)
    assert probe.probe_read_weights(str(py_file).encode(), ctypes.c_void_p(back.ctypes.data), ctypes.c_size_t(n), *_layout_args(), ctypes.c_float(0.33),
                                    err, ctypes.c_size_t(1024)) == 0, err.value
    assert back.tobytes() == params.tobytes()
    # another scene scale (metadata) and a non-finite value are both refused
    assert probe.probe_read_weights(str(py_file).encode(), ctypes.c_void_p(back.ctypes.data), ctypes.c_size_t(n), *_layout_args(), ctypes.c_float(0.5),
                                    err, ctypes.c_size_t(1024)) == 1
    assert b"does not match" in err.value
    params[5] = np.nan
    ngp_weights.export_weights(py_file, params, layout, 0.33)
    assert probe.probe_read_weights(str(py_file).encode(), ctypes.c_void_p(back.ctypes.data), ctypes.c_size_t(n), *_layout_args(), ctypes.c_float(0.33),
                                    err, ctypes.c_size_t(1024)) == 1
    assert b"non-finite" in err.value


@pytest.mark.parametrize("text,want", [('{ "b" : [1, 2], "a":{"y":"v","x":"w"} }', '{"a":{"x":"w","y":"v"},"b":[1,2]}'),
                                       ('{"k":"q\\"uote"}', '{"k":"q\\"uote"}')])
def test_header_canonical_form(probe, text, want):
    buf, err = ctypes.create_string_buffer(1024), _err()
    assert probe.probe_canonical(text.encode(), buf, ctypes.c_size_t(1024), err, ctypes.c_size_t(1024)) == 0, err.value
    assert buf.value.decode() == want


@pytest.mark.parametrize("bad", ['{"a":1,"a":2}', '{"a":01}', '{"a":-1}', '{"a":1} x', '{"a":"u\\u0041"}'])
def test_header_reader_rejects(probe, bad):
    buf, err = ctypes.create_string_buffer(1024), _err()
    assert probe.probe_canonical(bad.encode(), buf, ctypes.c_size_t(1024), err, ctypes.c_size_t(1024)) == 1


def _decode_png(data: bytes):
    assert data[:8] == b"\x89PNG\r\n\x1a\n"
    pos, idat = 8, b""
    w = h = None
    while pos < len(data):
        (length,) = struct.unpack(">I", data[pos:pos + 4])
        kind, body = data[pos + 4:pos + 8], data[pos + 8:pos + 8 + length]
        (crc,) = struct.unpack(">I", data[pos + 8 + length:pos + 12 + length])
        assert crc == zlib.crc32(kind + body) & 0xFFFFFFFF
        if kind == b"IHDR":
            w, h = struct.unpack(">II", body[:8])
            assert body[8:] == bytes([8, 2, 0, 0, 0])
        elif kind == b"IDAT":
            idat += body
        pos += 12 + length
    raw = zlib.decompress(idat)
    rows = np.frombuffer(raw, np.uint8).reshape(h, 1 + 3 * w)
    assert (rows[:, 0] == 0).all()
    return rows[:, 1:].reshape(h, w, 3)


@pytest.mark.parametrize("w,h", [(1, 1), (37, 5), (300, 90)])
def test_png_decodes_to_the_pixels(probe, tmp_path, w, h):
    rgb = np.random.default_rng(w * h).integers(0, 256, (h, w, 3), dtype=np.uint8)
    path, err = tmp_path / "x.png", _err()
    assert probe.probe_write_png(str(path).encode(), ctypes.c_void_p(rgb.ctypes.data), ctypes.c_uint32(w), ctypes.c_uint32(h), err,
                                 ctypes.c_size_t(1024)) == 0, err.value
    assert (_decode_png(path.read_bytes()) == rgb).all()


def test_constructor_errors_are_runtime_errors(probe):
    err = _err()
    assert probe.probe_construct_error(1, err, ctypes.c_size_t(1024)) == 1
    assert b"no training images" in err.value
    import torch

    if not torch.cuda.is_available():  # no device: the trainer's set-up fails and says why
        assert probe.probe_construct_error(0, err, ctypes.c_size_t(1024)) == 1
        assert err.value


@pytest.mark.gpu
def test_instant_ngp_lifecycle_through_cpp_api(probe, tmp_path):
    scene = workloads.procedural_dataset(n_train=8, n_test=2, width=96, height=96, seed=17)
    tr, te = scene["train"], scene["test"]
    px, cam = np.ascontiguousarray(tr["pixels"]), np.ascontiguousarray(tr["camera"], np.float32)
    tpx, tcam = np.ascontiguousarray(te["pixels"]), np.ascontiguousarray(te["camera"], np.float32)
    intr = np.array([tr["focal"][0], tr["focal"][1], tr["principal"][0], tr["principal"][1]], np.float32)
    res, err = np.zeros(6, np.float64), _err()
    P = lambda a: ctypes.c_void_p(a.ctypes.data)  # noqa: E731
    rc = probe.probe_lifecycle(ctypes.c_uint32(96), ctypes.c_uint32(96), ctypes.c_uint32(px.shape[0]), P(px), P(cam), ctypes.c_uint32(tpx.shape[0]),
                               P(tpx), P(tcam), P(intr), ctypes.c_int32(100), str(tmp_path).encode(), P(res), err, ctypes.c_size_t(1024))
    assert rc == 0, err.value
    loss, vpsnr, tpsnr, images, same, step = res
    assert np.isfinite(loss) and loss > 0 and step == 100
    assert 10.0 < vpsnr < 80.0 and 10.0 < tpsnr < 80.0
    assert images == 2 and same == 1.0
    for i in range(2):
        img = _decode_png((tmp_path / "test" / f"test_{i:04d}.png").read_bytes())
        assert img.shape == (96, 192, 3) and img.max() > 0
