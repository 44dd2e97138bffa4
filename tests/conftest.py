"""Shared pytest setup: the `gpu` marker, import paths, seeded input helpers."""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(REPO, "fused-logprob-entropy-cuda-kernel-for-llm-post-training_b200")
for p in (REPO, PKG_ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA GPU in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(autouse=True, scope="module")
def _kernel_waits_never_ran_out():
    """After every test module that used the GPU: no bounded wait inside a K1 kernel ran
    out (the kernels report that in a device word instead of hanging; read and cleared
    here, so a timeout anywhere fails the suite)."""
    yield
    try:
        import torch
        if not (torch.cuda.is_available() and torch.cuda.is_initialized()):
            return
        from kernel_opt import _C
    except Exception:  # pragma: no cover
        return
    status = _C.ring_status()
    assert status == 0, f"a bounded wait inside a K1 kernel ran out (status {status})"
