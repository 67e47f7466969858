"""Shared pytest setup: the `gpu` marker, import paths and common fixtures."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT / "instant-ngp_b200", ROOT / "oracle"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def oracle():
    from oracle import Oracle, build_oracle

    build_oracle()
    return Oracle()


@pytest.fixture(scope="session")
def ngp():
    import ngp_b200

    ngp_b200.lib()
    return ngp_b200


@pytest.fixture(scope="session")
def reflib():
    from oracle import RefLib

    return RefLib()
