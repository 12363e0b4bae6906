"""C-ABI checks that need no GPU: libds_kernels_sm100.so loads, exports exactly the entry
points include/ds_kernels.h declares, the ctypes table matches them, the host-only queries
work, and argument validation fails with the documented status before touching CUDA."""
import ctypes
import os
import re
import subprocess

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "ds_kernels.h")


def _declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"DS_API\s+[\w\s\*]+?\b(ds_\w+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    import ds_kernels
    lib = ds_kernels.library()
    names = _declared()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), n
    out = subprocess.run(["nm", "-D", "--defined-only", ds_kernels.LIBRARY_PATH],
                         capture_output=True, text=True, check=True).stdout
    exported = sorted({l.split()[-1] for l in out.splitlines() if re.search(r" T ds_", l)})
    assert exported == names


def test_ctypes_table_matches_header():
    import ds_kernels
    assert sorted(ds_kernels.SIGNATURES) == _declared()
    text = open(HEADER).read()
    for name, (_, args) in ds_kernels.SIGNATURES.items():
        m = re.search(r"DS_API\s+[\w\s\*]+?\b%s\s*\(([^)]*)\)" % name, text)
        assert m, name
        params = [p for p in m.group(1).split(",") if p.strip() and p.strip() != "void"]
        assert len(params) == len(args), name


def test_version_and_empty_last_error():
    import ds_kernels
    assert "sm_100a" in ds_kernels.version()


def test_workspace_queries_are_host_only():
    import ds_kernels
    lib = ds_kernels.library()
    assert lib.ds_moe_dispatch_workspace_size(16384, 64, 6) >= 16384 * 6 * 4
    assert lib.ds_moe_combine_workspace_size(98304, 16384) >= 98304 * 4
    ws = lib.ds_moe_layer_workspace_size(8192, 2048, 64, 6, 1408, 2816)
    S = 8192 * 6
    assert ws >= 2 * S * 2048 * 2 + S * 1408 * 2  # dispatched + expert out + h
    assert ws % 256 == 0


@pytest.mark.parametrize("call,code", [
    (lambda L: L.ds_moe_routing(None, None, None, None, 4, 65, 6, None), 1),
    (lambda L: L.ds_moe_routing(None, None, None, None, 4, 64, 9, None), 1),
    (lambda L: L.ds_moe_scan(None, None, 0, None), 1),
    (lambda L: L.ds_swiglu(None, None, 4, 7, None), 1),
    (lambda L: L.ds_moe_gemm1(None, None, None, None, 8, 64, 2048, 2000, None), 1),
    (lambda L: L.ds_moe_gemm2(None, None, None, None, 8, 64, 1408, 2000, None), 1),
    (lambda L: L.ds_kv_upproj(None, None, None, 8, 512, 100, None), 1),
    (lambda L: L.ds_rope(None, None, None, None, None, None, 1, 16, 4, 63, None), 1),
    (lambda L: L.ds_rms_norm(None, None, None, 4, 511, ctypes.c_float(1e-6), None), 1),
    (lambda L: L.ds_moe_combine(None, None, None, None, 6, 2048, 0, None, 0, None), 1),
    (lambda L: L.ds_moe_dispatch(None, None, None, None, None, None, None, 4, 2047, 64, 6,
                                 None, 0, None), 1),
    # the persistent attention kernel's work counter lives in the workspace: none, or too
    # small, is refused before anything touches the device
    (lambda L: L.ds_mla_attention(ctypes.c_void_p(256), 3648, ctypes.c_void_p(512),
                                  ctypes.c_void_p(768), 1, 128, 16, ctypes.c_float(0.1), None,
                                  256, None), 1),
    (lambda L: L.ds_mla_attention(ctypes.c_void_p(256), 3648, ctypes.c_void_p(512),
                                  ctypes.c_void_p(768), 1, 128, 16, ctypes.c_float(0.1),
                                  ctypes.c_void_p(1024), 128, None), 1),
])
def test_argument_validation_without_gpu(call, code):
    import ds_kernels
    lib = ds_kernels.library()
    assert call(lib) == code
    assert lib.ds_last_error().decode()


def test_mla_attention_workspace_is_the_tile_counter():
    import ds_kernels
    assert ds_kernels.library().ds_mla_attention_workspace_size(4, 4096, 16) == 256


def test_zero_size_calls_are_no_ops_without_gpu():
    import ds_kernels
    lib = ds_kernels.library()
    assert lib.ds_swiglu(None, None, 0, 1408, None) == 0
    assert lib.ds_moe_gemm1(None, None, None, None, 0, 64, 2048, 2816, None) == 0
    assert lib.ds_moe_gemm2(None, None, None, None, 0, 64, 1408, 2048, None) == 0
    assert lib.ds_kv_upproj(None, None, None, 0, 512, 4096, None) == 0
