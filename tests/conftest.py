"""Shared pytest setup.

Import contract (mirrors the reference tests, which put src/kernels and build/ on sys.path):
the package directory `deepseek-v2-lite-cuda_b200/` is put on sys.path so that
`import ds_kernels`, `from moe_fused import FusedMoELayer` and `import expert_prepack` work
exactly as in the reference's tests; the repo root is put on sys.path for `oracle`.

Tests marked `gpu` need a CUDA device (a B200); everything else runs on the CPU.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "deepseek-v2-lite-cuda_b200")
for p in (PKG, ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_cuda = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_cuda = False
    if has_cuda:
        return
    skip = pytest.mark.skip(reason="needs a CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN
