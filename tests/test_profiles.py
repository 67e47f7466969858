"""The committed ncu summaries (profiles/) name kernels this library defines and give commands that
run committed files only."""
from __future__ import annotations

import re

from conftest import ROOT


def _kernels() -> set[str]:
    names = set()
    for src in (ROOT / "instant-ngp_b200" / "csrc").glob("*.cu"):
        names |= set(re.findall(r"__global__\s+void\s+(?:__launch_bounds__\([^)]*\)\s+)?(\w+)", src.read_text()))
    return names


def test_profiles_name_existing_kernels_and_committed_commands():
    kernels = _kernels()
    summaries = sorted((ROOT / "profiles").glob("*.md"))
    assert summaries
    for md in summaries:
        text = md.read_text()
        stem = md.stem.split("__")[0]
        if stem.endswith("_kernel"):
            assert stem in kernels, f"{md.name}: no kernel {stem} in csrc"
        assert "_work" not in text, f"{md.name} names a working file"
        assert "```" in text and ("ncu " in text), f"{md.name} gives no ncu command"
