"""Seeded synthetic workloads standing in for the BASELINE configurations (numpy, host side).

The reference measures on NeRF-synthetic scenes that are not available here; these generators
produce inputs with the configurations' shapes, sizes and value distributions instead.  Every
generator takes a seed and returns host numpy arrays, so the CUDA library, the reference build
and the CPU oracle all see identical bytes.
"""
from __future__ import annotations

import math

import numpy as np


def encode_inputs(n: int, n_params: int, L: int, F: int, seed: int = 0, coord_stride: int = 3):
    """Config 0: n points uniform in [0,1)^3 (fp32 [n][coord_stride]), a U(-1e-4, 1e-4) fp16 table
    and dL/dy ~ N(0,1) rounded to fp16 in the feature-major [L*F][n] layout."""
    rng = np.random.default_rng(seed)
    coords = np.zeros((n, coord_stride), np.float32)
    coords[:, :3] = rng.random((n, 3), dtype=np.float32)
    if coord_stride >= 7:
        coords[:, 3] = math.sqrt(3.0) / 1024.0
        coords[:, 4:7] = 0.5
    table = (rng.random(n_params, dtype=np.float32) * 2e-4 - 1e-4).astype(np.float16)
    dy = rng.standard_normal((L * F, n), dtype=np.float32).astype(np.float16)
    return coords, table, dy


def xavier_mlp_params(seed: int = 0) -> np.ndarray:
    """Config 1: the 10,240 packed MLP weights, Xavier-uniform per matrix (fan_in + fan_out), fp16,
    in the reference's order and shapes (ngp.train.cu:1429-1452)."""
    rng = np.random.default_rng(seed)
    shapes = [(64, 32), (16, 64), (64, 32), (64, 64), (16, 64)]
    parts = []
    for out_dim, in_dim in shapes:
        s = math.sqrt(6.0 / (out_dim + in_dim))
        parts.append(rng.uniform(-s, s, size=out_dim * in_dim).astype(np.float32))
    return np.concatenate(parts).astype(np.float16)


def mlp_inputs(n: int, seed: int = 0):
    """Config 1: n rows of encoded inputs U(-1, 1) fp16 [32][n], sample records whose view
    directions are uniform on S^2 (z = 1 - 2u, phi = 2 pi v), and dL/d(output) fp16 [n][16]
    (channels 0-3 ~ N(0, 1), the rest zero)."""
    rng = np.random.default_rng(seed)
    x = rng.uniform(-1.0, 1.0, size=(32, n)).astype(np.float16)
    u, v = rng.random(n), rng.random(n)
    z = 1.0 - 2.0 * u
    r = np.sqrt(np.maximum(0.0, 1.0 - z * z))
    phi = 2.0 * math.pi * v
    d = np.stack([r * np.cos(phi), r * np.sin(phi), z], axis=1)
    coords = np.zeros((n, 7), np.float32)
    coords[:, :3] = rng.random((n, 3))
    coords[:, 3] = math.sqrt(3.0) / 1024.0
    coords[:, 4:7] = ((d + 1.0) * 0.5).astype(np.float32)
    dy = np.zeros((n, 16), np.float16)
    dy[:, :4] = rng.standard_normal((n, 4)).astype(np.float16)
    return x, coords, dy


# ---------------------------------------------------------------------------------------------
# Config 3/4: procedural scene (64 Lambert spheres) and its camera conventions
# ---------------------------------------------------------------------------------------------
DEFAULT_SCENE_SCALE = 0.33  # ngp.dataset.ixx:5
SCENE_OFFSET = 0.5          # ngp.dataset.cpp:10


def look_at_c2w(position: np.ndarray) -> np.ndarray:
    """OpenGL-convention camera-to-world 4x4 (x right, y up, z back) looking at the origin, world up +z."""
    z = position / np.linalg.norm(position)
    up = np.array([0.0, 0.0, 1.0])
    if abs(z @ up) > 0.999:
        up = np.array([0.0, 1.0, 0.0])
    x = np.cross(up, z)
    x /= np.linalg.norm(x)
    y = np.cross(z, x)
    m = np.eye(4)
    m[:3, 0], m[:3, 1], m[:3, 2], m[:3, 3] = x, y, z, position
    return m


def nerf_to_ngp_camera(c2w: np.ndarray, scene_scale: float = DEFAULT_SCENE_SCALE) -> np.ndarray:
    """The reference's NeRF-synthetic camera conversion (ngp.dataset.cpp:47-65): flip the y and z
    axes, scale and offset the position into the unit cube, then permute the axes (x, y, z) ->
    (y, z, x).  Returns 12 floats: three axis columns and the origin."""
    cam = np.array(c2w, np.float32)[:3, :4].T.copy()  # cam[c] = column c
    cam[1] = -cam[1]
    cam[2] = -cam[2]
    cam[3] = cam[3] * np.float32(scene_scale) + np.float32(SCENE_OFFSET)
    out = np.empty(12, np.float32)
    for c in range(4):
        out[3 * c: 3 * c + 3] = (cam[c][1], cam[c][2], cam[c][0])
    return out


def hemisphere_positions(n: int, radius: float, rng) -> np.ndarray:
    z = rng.uniform(0.15, 1.0, n)
    phi = rng.uniform(0.0, 2.0 * math.pi, n)
    r = np.sqrt(1.0 - z * z)
    return np.stack([r * np.cos(phi), r * np.sin(phi), z], axis=1) * radius


def sphere_scene(seed: int = 3, n_spheres: int = 64):
    rng = np.random.default_rng(seed)
    return {"centers": rng.uniform(-1.0, 1.0, (n_spheres, 3)), "radii": rng.uniform(0.05, 0.4, n_spheres),
            "albedo": rng.uniform(0.15, 1.0, (n_spheres, 3)), "light": np.array([0.4, 0.3, 0.866]) / np.linalg.norm([0.4, 0.3, 0.866])}


def render_spheres(scene: dict, c2w: np.ndarray, width: int, height: int, focal: float, device: str = "cpu") -> np.ndarray:
    """Analytic ray-traced RGBA8 image of the sphere scene (Lambert shading + 0.1 ambient, alpha 0
    where no sphere is hit), rendered with torch on `device`."""
    import torch

    dev = torch.device(device)
    c2w_t = torch.tensor(c2w, dtype=torch.float64, device=dev)
    v, u = torch.meshgrid(torch.arange(height, device=dev, dtype=torch.float64), torch.arange(width, device=dev, dtype=torch.float64), indexing="ij")
    d_cam = torch.stack([(u + 0.5 - width * 0.5) / focal, -(v + 0.5 - height * 0.5) / focal, -torch.ones_like(u)], dim=-1).reshape(-1, 3)
    d = d_cam @ c2w_t[:3, :3].T
    d = d / d.norm(dim=1, keepdim=True)
    o = c2w_t[:3, 3]
    C = torch.tensor(scene["centers"], dtype=torch.float64, device=dev)
    R = torch.tensor(scene["radii"], dtype=torch.float64, device=dev)
    oc = o[None, :] - C  # [S,3]
    b = d @ oc.T  # [P,S]
    c = (oc * oc).sum(1) - R * R
    disc = b * b - c[None, :]
    t = -b - torch.sqrt(torch.clamp(disc, min=0.0))
    t = torch.where((disc > 0) & (t > 1e-6), t, torch.full_like(t, float("inf")))
    tmin, idx = t.min(dim=1)
    hit = torch.isfinite(tmin)
    p = o[None, :] + d * torch.where(hit, tmin, torch.zeros_like(tmin))[:, None]
    n = (p - C[idx]) / R[idx][:, None]
    L = torch.tensor(scene["light"], dtype=torch.float64, device=dev)
    shade = 0.1 + 0.9 * torch.clamp(n @ L, min=0.0)
    rgb = torch.tensor(scene["albedo"], dtype=torch.float64, device=dev)[idx] * shade[:, None]
    rgba = torch.zeros((d.shape[0], 4), dtype=torch.float64, device=dev)
    rgba[:, :3] = torch.where(hit[:, None], rgb, torch.zeros_like(rgb))
    rgba[:, 3] = hit.double()
    return (rgba.clamp(0, 1) * 255.0 + 0.5).to(torch.uint8).reshape(height, width, 4).cpu().numpy()


def procedural_dataset(n_train: int = 100, n_test: int = 20, width: int = 800, height: int = 800, fov_x: float = 0.69, seed: int = 3,
                       n_validation: int = 0, device: str = "cpu", scene_scale: float = DEFAULT_SCENE_SCALE) -> dict:
    """Config 3: the 64-sphere scene seen from cameras on a radius-4 hemisphere looking at the
    origin (horizontal FOV 0.69 rad), converted with the reference's camera convention."""
    scene = sphere_scene(seed)
    rng = np.random.default_rng(seed + 1)
    focal = 0.5 * width / math.tan(fov_x * 0.5)
    out = {}
    for name, count in (("train", n_train), ("validation", n_validation), ("test", n_test)):
        if count == 0:
            out[name] = None
            continue
        pos = hemisphere_positions(count, 4.0, rng)
        pixels = np.zeros((count, height, width, 4), np.uint8)
        cams = np.zeros((count, 12), np.float32)
        for i in range(count):
            c2w = look_at_c2w(pos[i])
            pixels[i] = render_spheres(scene, c2w, width, height, focal, device)
            cams[i] = nerf_to_ngp_camera(c2w, scene_scale)
        out[name] = {"pixels": pixels, "camera": cams, "focal": (focal, focal), "principal": (width * 0.5, height * 0.5)}
    return out


def render_poses(n: int = 64, width: int = 1920, height: int = 1080, fov_x: float = 0.69, seed: int = 4,
                 scene_scale: float = DEFAULT_SCENE_SCALE) -> dict:
    """Config 4 novel views: n poses on the radius-4 sphere looking at the origin, width x height,
    horizontal FOV 0.69 rad, in the reference's camera convention."""
    rng = np.random.default_rng(seed)
    v = rng.standard_normal((n, 3))
    pos = 4.0 * v / np.linalg.norm(v, axis=1, keepdims=True)
    cams = np.stack([nerf_to_ngp_camera(look_at_c2w(p), scene_scale) for p in pos]).astype(np.float32)
    focal = 0.5 * width / math.tan(fov_x * 0.5)
    return {"camera": cams, "width": width, "height": height, "focal": (focal, focal), "principal": (width * 0.5, height * 0.5)}


def march_rays_config2(n: int = 1 << 18, seed: int = 2) -> np.ndarray:
    """Config 2 rays in the unit-cube frame: origins uniform on the radius-4 sphere (world), aimed
    at the origin plus U(-0.1, 0.1)^3 jitter, normalised on the host, world -> unit x/3 + 0.5."""
    rng = np.random.default_rng(seed)
    v = rng.standard_normal((n, 3))
    o = 4.0 * v / np.linalg.norm(v, axis=1, keepdims=True)
    tgt = rng.uniform(-0.1, 0.1, (n, 3))
    d = tgt - o
    d /= np.linalg.norm(d, axis=1, keepdims=True)
    rays = np.zeros((n, 6), np.float32)
    rays[:, :3] = (o / 3.0 + 0.5).astype(np.float32)
    rays[:, 3:] = d.astype(np.float32)
    return rays


def gaussian_blob_density(n_blobs: int = 8, seed: int = 2):
    """Config 2 density field: sum of 8 isotropic Gaussians (centres in [-1,1]^3, sigma in
    [0.05, 0.3], amplitude in [10, 100]) in world coordinates."""
    rng = np.random.default_rng(seed + 100)
    return {"c": rng.uniform(-1, 1, (n_blobs, 3)), "s": rng.uniform(0.05, 0.3, n_blobs), "a": rng.uniform(10, 100, n_blobs)}


def blob_grid_values(blobs: dict) -> np.ndarray:
    """Optical thickness density * dt of the blob field at the 128^3 cell centres, in the grid's
    Morton order (cell x,y,z over the unit cube; world = (unit - 0.5) * 3)."""
    g = (np.arange(128) + 0.5) / 128.0
    X, Y, Z = np.meshgrid(g, g, g, indexing="ij")
    P = (np.stack([X, Y, Z], -1).reshape(-1, 3) - 0.5) * 3.0
    dens = np.zeros(P.shape[0])
    for c, s, a in zip(blobs["c"], blobs["s"], blobs["a"]):
        dens += a * np.exp(-((P - c) ** 2).sum(1) / (2 * s * s))
    thick = (dens * (math.sqrt(3.0) / 1024.0)).astype(np.float32)
    idx = np.arange(128 ** 3)
    x, y, z = idx // (128 * 128), (idx // 128) % 128, idx % 128

    def spread(v):
        v = v.astype(np.uint64)
        out = np.zeros_like(v)
        for b in range(7):
            out |= ((v >> b) & 1) << (3 * b)
        return out

    morton = spread(x) | (spread(y) << 1) | (spread(z) << 2)
    vals = np.zeros(128 ** 3, np.float32)
    vals[morton.astype(np.int64)] = thick
    return vals


def eval_composite_inputs(width: int = 64, height: int = 48, n_images: int = 2, max_steps: int = 40, seed: int = 0):
    """Inputs of evaluation compositing for every pixel of image 1: per-pixel (count, base) with
    counts in [0, max_steps] and ragged bases, sample records whose dt is U(0.5, 8) x sqrt(3)/1024,
    raw network outputs ~ N(0, 2) fp16 [samples][16] (density raw N(2, 2)), and RGBA8 target
    images with a mix of opaque, transparent and partial alpha."""
    rng = np.random.default_rng(seed)
    n = width * height
    counts = rng.integers(0, max_steps + 1, n).astype(np.uint32)
    counts[rng.random(n) < 0.1] = 0
    gaps = rng.integers(0, 3, n).astype(np.uint32)
    bases = (np.cumsum(counts + gaps) - counts).astype(np.uint32)
    total = int(bases[-1] + counts[-1]) + 1
    numsteps = np.stack([counts, bases], axis=1).astype(np.uint32)
    coords = np.zeros((total, 7), np.float32)
    coords[:, :3] = rng.random((total, 3), dtype=np.float32)
    coords[:, 3] = (rng.uniform(0.5, 8.0, total) * math.sqrt(3.0) / 1024.0).astype(np.float32)
    coords[:, 4:7] = rng.random((total, 3), dtype=np.float32)
    out = rng.normal(0.0, 2.0, (total, 16)).astype(np.float16)
    out[:, 3] = rng.normal(2.0, 2.0, total).astype(np.float16)
    pixels = rng.integers(0, 256, (n_images, height, width, 4)).astype(np.uint8)
    alpha = pixels[..., 3]
    alpha[rng.random(alpha.shape) < 0.3] = 0
    alpha[rng.random(alpha.shape) < 0.3] = 255
    return numsteps, coords, out, pixels
