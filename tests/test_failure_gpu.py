"""Host-side fault injection through the C ABI on one GPU (no GPU fault is raised: the library
reports an injected error status where a failing CUDA call would).  The reference's contract
(ngp.train.cu:1290, ngp.train.cpp:152-154): a failed device call surfaces as an error with a
message, and the trainer stays destroyable; a new trainer works afterwards."""
from __future__ import annotations

import pytest

import workloads

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def scene():
    return workloads.procedural_dataset(n_train=4, n_test=1, width=64, height=64, seed=5)


def test_injected_allocation_failure_fails_construction(ngp, scene):
    ngp.fault_inject("alloc", 3)
    try:
        with pytest.raises(RuntimeError, match="injected fault \\(alloc\\)"):
            ngp.InstantNGP(scene, ngp.config0_trainer_config())
    finally:
        ngp.fault_inject("alloc", 0)
    model = ngp.InstantNGP(scene, ngp.config0_trainer_config())
    assert model.train(2)["measured_sample_count"] > 0
    model.close()


def test_injected_launch_failure_fails_the_step(ngp, scene):
    model = ngp.InstantNGP(scene, ngp.config0_trainer_config())
    model.train(1)
    ngp.fault_inject("launch", 7)
    try:
        with pytest.raises(RuntimeError, match="injected fault \\(launch\\)"):
            model.train(3)
    finally:
        ngp.fault_inject("launch", 0)
    model.close()
    fresh = ngp.InstantNGP(scene, ngp.config0_trainer_config())
    st = fresh.train(3)
    assert st["measured_sample_count"] > 0 and st["step"] == 3
    fresh.close()
