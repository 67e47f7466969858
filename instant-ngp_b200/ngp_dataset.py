"""Scene loaders: the reference's NeRF-synthetic and DD-NeRF formats (ngp.dataset.cpp:12-190,
ngp.dataset.ixx:7-25), producing the split dicts `InstantNGP` takes.

A split is ``{"pixels": uint8 [F][H][W][4], "camera": float32 [F][12], "focal": (fx, fy),
"principal": (cx, cy)}``; the dataset dict holds "train", "validation", "test" and
"scene_scale".  Cameras are converted exactly as the reference does (float32 arithmetic): the
transform matrix is read column by column, columns 1 and 2 are negated, the position is scaled
by the scene scale and offset by 0.5, then the axes are permuted (x, y, z) -> (y, z, x) into 12
floats (three axis columns and the origin).  Images are decoded to RGBA8 (stbi_load with 4
components in the reference; here Pillow, identical bytes for 8-bit PNG).  All frames of a split
must share one size, as the trainer keeps one resolution per split.
"""
from __future__ import annotations

import json
import math
from pathlib import Path

import numpy as np

DEFAULT_SCENE_SCALE = 0.33  # ngp.dataset.ixx:5
SCENE_OFFSET = 0.5          # ngp.dataset.cpp:10


def _load_rgba(path: Path) -> np.ndarray:
    from PIL import Image

    if not path.is_file():
        raise RuntimeError(f"failed to load image '{path}'.")
    with Image.open(path) as im:
        rgba = np.asarray(im.convert("RGBA"), dtype=np.uint8)
    if rgba.shape[0] == 0 or rgba.shape[1] == 0:
        raise RuntimeError(f"image '{path}' has invalid dimensions.")
    return rgba


def ngp_camera(transform_matrix, scene_scale: float) -> np.ndarray:
    """12-float camera of one frame (ngp.dataset.cpp:47-65), in float32."""
    m = np.asarray(transform_matrix, dtype=np.float32)
    if m.shape != (4, 4):
        raise RuntimeError("transform_matrix must be 4x4.")
    cam = m.T.copy()  # cam[column][row]
    cam[1] = -cam[1]
    cam[2] = -cam[2]
    s, o = np.float32(scene_scale), np.float32(SCENE_OFFSET)
    for r in range(3):
        cam[3][r] = np.float32(np.float32(cam[3][r] * s) + o)
    row0 = [cam[0][0], cam[1][0], cam[2][0], cam[3][0]]
    row1 = [cam[0][1], cam[1][1], cam[2][1], cam[3][1]]
    row2 = [cam[0][2], cam[1][2], cam[2][2], cam[3][2]]
    return np.array([row1[0], row2[0], row0[0], row1[1], row2[1], row0[1], row1[2], row2[2], row0[2], row1[3], row2[3], row0[3]], np.float32)


def _split(frames: list, what: str) -> dict:
    if not frames:
        return None
    h, w = frames[0]["rgba"].shape[:2]
    for f in frames:
        if f["rgba"].shape[:2] != (h, w):
            raise RuntimeError(f"{what}: every frame of a split must have the same size")
        if (f["focal"], f["principal"]) != (frames[0]["focal"], frames[0]["principal"]):
            raise RuntimeError(f"{what}: every frame of a split must share the intrinsics")
    return {"pixels": np.stack([f["rgba"] for f in frames]), "camera": np.stack([f["camera"] for f in frames]),
            "focal": frames[0]["focal"], "principal": frames[0]["principal"]}


def _nerf_synthetic_split(root: Path, file_name: str, scene_scale: float) -> list:
    json_path = root / file_name
    meta = json.loads(json_path.read_text())
    angle = np.float32(meta["camera_angle_x"])
    frames = []
    for fj in meta["frames"]:
        p = Path(fj["file_path"])
        if p.suffix == "":
            p = p.with_suffix(".png")
        if not p.is_absolute():
            p = json_path.parent / p
        rgba = _load_rgba(Path(str(p)).resolve())
        h, w = rgba.shape[:2]
        focal = float(np.float32(np.float32(0.5) * np.float32(w)) / np.float32(math.tan(float(angle * np.float32(0.5)))))
        frames.append({"rgba": rgba, "camera": ngp_camera(fj["transform_matrix"], scene_scale), "focal": (focal, focal),
                       "principal": (float(np.float32(w) * np.float32(0.5)), float(np.float32(h) * np.float32(0.5)))})
    return frames


def load_nerf_synthetic(path, scene_scale: float = DEFAULT_SCENE_SCALE) -> dict:
    """transforms_{train,val,test}.json + images (ngp.dataset.cpp:12-93)."""
    if not math.isfinite(scene_scale) or scene_scale <= 0.0:
        raise RuntimeError("scene scale must be finite and positive.")
    root = Path(path)
    return {"train": _split(_nerf_synthetic_split(root, "transforms_train.json", scene_scale), "train"),
            "validation": _split(_nerf_synthetic_split(root, "transforms_val.json", scene_scale), "validation"),
            "test": _split(_nerf_synthetic_split(root, "transforms_test.json", scene_scale), "test"),
            "scene_scale": float(np.float32(scene_scale))}


def fnv1a64(text: str) -> int:
    """64-bit FNV-1a of the UTF-8 bytes (the DD-NeRF split hash, ngp.dataset.cpp:131-136)."""
    h = 14695981039346656037
    for b in text.encode():
        h ^= b
        h = (h * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


def load_dd_nerf(path, scene_scale: float = DEFAULT_SCENE_SCALE) -> dict:
    """cameras.json + images/ with a hash split: FNV-1a of the file name % 10 == 0 -> test,
    == 1 -> validation, else train (ngp.dataset.cpp:107-187)."""
    if not math.isfinite(scene_scale) or scene_scale <= 0.0:
        raise RuntimeError("scene scale must be finite and positive.")
    root = Path(path)
    json_path = root / "cameras.json"
    if not json_path.is_file():
        raise RuntimeError(f"DD-NeRF dataset '{root}' is missing cameras.json.")
    if not (root / "images").is_dir():
        raise RuntimeError(f"DD-NeRF dataset '{root}' is missing an images directory.")
    meta = json.loads(json_path.read_text())
    frames_json = meta["frames"]
    w, h = int(meta["w"]), int(meta["h"])
    fx, fy, cx, cy = (float(np.float32(meta[k])) for k in ("fl_x", "fl_y", "cx", "cy"))
    if not isinstance(frames_json, list) or not frames_json:
        raise RuntimeError("DD-NeRF cameras.json must contain a non-empty frames array.")
    if w == 0 or h == 0:
        raise RuntimeError("DD-NeRF cameras.json declares invalid image dimensions.")
    if not all(math.isfinite(v) for v in (fx, fy)) or fx <= 0 or fy <= 0:
        raise RuntimeError("DD-NeRF cameras.json declares invalid focal lengths.")
    if not (0 <= cx < w and 0 <= cy < h):
        raise RuntimeError("DD-NeRF cameras.json declares an invalid principal point.")
    splits = {"train": [], "validation": [], "test": []}
    for fj in frames_json:
        name = Path(fj["file_path"]).name
        p = Path(fj["file_path"])
        if not p.is_absolute():
            p = root / p
        if not p.is_file():
            raise RuntimeError(f"DD-NeRF image '{p}' does not exist.")
        rgba = _load_rgba(p)
        if rgba.shape[:2] != (h, w):
            raise RuntimeError(f"DD-NeRF image '{p}' is {rgba.shape[1]}x{rgba.shape[0]} but cameras.json declares {w}x{h}.")
        frame = {"rgba": rgba, "camera": ngp_camera(fj["transform_matrix"], scene_scale), "focal": (fx, fy), "principal": (cx, cy)}
        k = fnv1a64(name) % 10
        splits["test" if k == 0 else "validation" if k == 1 else "train"].append(frame)
    for name, frames in splits.items():
        if not frames:
            raise RuntimeError(f"DD-NeRF split produced no {'training' if name == 'train' else name} frames.")
    return {name: _split(frames, name) for name, frames in splits.items()} | {"scene_scale": float(np.float32(scene_scale))}


def load_dataset(path, scene_scale: float = DEFAULT_SCENE_SCALE) -> tuple[dict, str]:
    """Detect the format as the reference's CLI does (main.cpp): exactly one of the NeRF-synthetic
    transforms_*.json set or DD-NeRF cameras.json + images/."""
    root = Path(path)
    synthetic = all((root / f"transforms_{s}.json").is_file() for s in ("train", "val", "test"))
    dd = (root / "cameras.json").is_file() and (root / "images").is_dir()
    if synthetic == dd:
        raise RuntimeError(f"dataset path '{root}' must contain exactly one supported dataset marker set: NeRF synthetic transforms_*.json "
                           "or DD-NeRF cameras.json + images/.")
    return (load_nerf_synthetic(root, scene_scale), "nerf-synthetic") if synthetic else (load_dd_nerf(root, scene_scale), "dd-nerf-dataset")
