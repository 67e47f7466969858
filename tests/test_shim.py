"""The drop-in `ngp::cuda` layer on the CPU: it compiles against the reference's own ngp.train.h
and defines every function that header declares (checked when the reference sources are present;
the GPU tier runs the reference's training loop on it)."""
from __future__ import annotations

import re
import subprocess
from pathlib import Path

import pytest

from oracle import reference_dir

ROOT = Path(__file__).resolve().parents[1]
REF = reference_dir()
REF_HEADER = REF / "ngp.train.h" if REF is not None else Path("ngp.train.h.absent")


@pytest.mark.skipif(not REF_HEADER.exists(), reason="reference sources not present")
def test_drop_in_layer_defines_every_declared_function():
    subprocess.run(["make", "-s", "-C", str(ROOT / "oracle"), f"REF_DIR={REF}", "shim"], check=True)
    so = ROOT / "oracle" / "_ref" / "libngp_shim_replay.so"
    names = set(re.findall(r"\bvoid\s+(\w+)\s*\(", re.sub(r"template\s*<[^>]*>[^{]*\{[^}]*\}[^}]*\}", "", REF_HEADER.read_text())))
    assert len(names) >= 25
    syms = subprocess.run(["nm", "-DC", "--defined-only", str(so)], capture_output=True, text=True, check=True).stdout
    defined = set(re.findall(r"ngp::cuda::(\w+)\(", syms))
    assert names <= defined, sorted(names - defined)
