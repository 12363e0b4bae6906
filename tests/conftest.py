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


def _record(max_abs, rel, ref_max, atol):
    """With DS_RECORD_ERRORS=<file>, append the check's max-abs and relative-L2 errors (and
    the reference's largest magnitude) as one JSON line per check, keyed by the test."""
    path = os.environ.get("DS_RECORD_ERRORS")
    if not path:
        return
    import json
    with open(path, "a") as f:
        f.write(json.dumps({"test": os.environ.get("PYTEST_CURRENT_TEST", "").split(" ")[0],
                            "max_abs": max_abs, "rel_l2": rel, "ref_max_abs": ref_max,
                            "atol": atol}) + "\n")


def assert_bf16_close(out, ref, atol, rel_l2_max=1e-2):
    """bf16 output vs f32 reference: |out - ref| <= atol + 2^-8 |ref| elementwise (2^-8 is the
    relative half-ulp of bf16 round-to-nearest, so large outputs are held to their own
    precision) and relative L2 error <= rel_l2_max."""
    import torch
    o = out.float().cpu()
    r = ref.float().cpu()
    err = (o - r).abs()
    bound = atol + (2.0 ** -8) * r.abs()
    worst = (err - bound).max().item()
    rel = (torch.linalg.vector_norm(o - r) / torch.linalg.vector_norm(r).clamp_min(1e-30)).item()
    _record(err.max().item(), rel, r.abs().max().item(), atol)
    assert worst <= 0 and rel <= rel_l2_max, (
        f"max excess over atol+2^-8|ref|: {worst:.3e}, max-abs {err.max().item():.3e}, rel-L2 {rel:.3e}")
