"""Build the in-tree CUDA library ``libngp_b200.so`` for sm_100a with nvcc.

Usage: ``python instant-ngp_b200/build.py [--force] [--jobs N]``.

The bench-only probes (``bench_probes/probes.cu``) build into their own library.

Each ``csrc/*.cu`` / ``csrc/*.cpp`` is compiled to an object under ``_build/`` (skipped when
the object is newer than the source and every header), then linked into
``instant-ngp_b200/libngp_b200.so`` next to this file.  The library is loaded from that path by
``ngp_b200.py``; it is never installed into site-packages.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libngp_b200.so"
PROBES_SRC = PKG / "bench_probes" / "probes.cu"
PROBES_LIB = PKG / "bench_probes" / "libngp_bench_probes.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden", "-I", str(ROOT / "include"), "-I", str(CSRC),
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted((ROOT / "include").glob("*.h"))


def _stale(obj: Path, src: Path, headers: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *headers])


def _compile(src: Path, force: bool, headers: list[Path]) -> Path:
    obj = BUILD / (src.name + ".o")
    if force or _stale(obj, src, headers):
        cmd = [nvcc(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        if src.suffix == ".cpp":
            cmd = [nvcc(), "-x", "cu", *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    return obj


def build(force: bool = False, jobs: int | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    headers = _headers()
    sources = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))
    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, headers), sources))
    if force or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart", "-lnccl"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
    build_probes(force)
    return LIB


def build_probes(force: bool = False) -> Path:
    """The bench-only probe library (bench_probes/libngp_bench_probes.so), separate from the
    product library; only bench.py loads it."""
    if force or not PROBES_LIB.exists() or PROBES_SRC.stat().st_mtime > PROBES_LIB.stat().st_mtime:
        cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "-shared",
               "-I", str(CSRC), "-o", str(PROBES_LIB), str(PROBES_SRC), "-lcudart"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {PROBES_SRC.name}:\n{res.stdout}\n{res.stderr}")
    return PROBES_LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    args = ap.parse_args()
    print(build(args.force, args.jobs))
    sys.exit(0)
