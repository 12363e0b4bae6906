"""The allocation-free dispatch entry point, ds_moe_dispatch_noalloc.

Callers that cannot allocate device memory where they dispatch (a serving loop keeping the
CUDA allocator off its hot path, a binding holding only plain pointers, code running during
another stream's graph capture) use this variant: its scratch is a fixed array inside the
library instead of a caller-provided workspace.  These tests call it through the C ABI and
check that it produces exactly what ds_moe_dispatch (the workspace entry point) produces —
dispatch is an integer permutation plus row copies, so the tolerance is zero — on two calls
in a row with different inputs (the shared array keeps the previous call's contents, which
must not leak into the next result), and that oversized calls are refused.

This file is named so that pytest collects it last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

E, K, H = 64, 6, 2048


def _lib():
    import ds_kernels
    return ds_kernels, ds_kernels.library()


def _inputs(T, seed):
    import ds_kernels
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(T, E, generator=g).cuda()
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).cuda()
    idx, w, counts = ds_kernels.moe_routing(logits, top_k=K)
    offsets = ds_kernels.moe_scan(counts)
    return x, idx, w, offsets


def _noalloc(lib, x, idx, w, offsets):
    T = x.shape[0]
    S = T * K
    disp = torch.full((S, H), float("nan"), dtype=torch.bfloat16, device="cuda")
    tmap = torch.full((S,), -7, dtype=torch.int32, device="cuda")
    dw = torch.full((S,), -1.0, dtype=torch.float32, device="cuda")
    st = lib.ds_moe_dispatch_noalloc(x.data_ptr(), idx.data_ptr(), w.data_ptr(), offsets.data_ptr(),
                                     disp.data_ptr(), tmap.data_ptr(), dw.data_ptr(), T, H, E, K,
                                     torch.cuda.current_stream().cuda_stream)
    assert st == 0, lib.ds_last_error().decode()
    return disp, tmap, dw


def test_noalloc_matches_workspace_dispatch_on_consecutive_calls():
    ds_kernels, lib = _lib()
    # The first call fills the whole scratch (exactly the largest accepted size: every
    # per-block histogram and every rank entry); the next ones are smaller and take the plan
    # kernel's looped path (more than 16 routing blocks) and then its short path, so stale
    # entries of a larger call must not leak into their results.
    for T, seed in ((65536, 1), (20000, 2), (777, 3)):
        x, idx, w, offsets = _inputs(T, seed)
        ref_disp, ref_tmap, ref_dw = ds_kernels.moe_dispatch(x, idx, w, offsets)
        disp, tmap, dw = _noalloc(lib, x, idx, w, offsets)
        torch.cuda.synchronize()
        assert torch.equal(tmap, ref_tmap), T
        assert torch.equal(dw, ref_dw), T
        assert torch.equal(disp, ref_disp), T
    assert ds_kernels.device_status() == ds_kernels.DS_OK


def test_noalloc_rejects_sizes_beyond_its_scratch():
    ds_kernels, lib = _lib()
    limit = 65536  # DS_NOALLOC_MAX_TOKENS
    st = lib.ds_moe_dispatch_noalloc(None, None, None, None, None, None, None, limit + 1, H, E, K,
                                     None)
    assert st == ds_kernels.DS_ERR_UNSUPPORTED
    assert "exceeds" in lib.ds_last_error().decode()


def test_noalloc_rejects_a_stream_of_another_device():
    """The scratch address is the current device's; a stream that belongs to another GPU is
    refused before anything is launched (needs two GPUs)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ds_kernels, lib = _lib()
    x, idx, w, offsets = _inputs(64, 4)
    other = torch.cuda.Stream(device=1)
    S = 64 * K
    disp = torch.empty((S, H), dtype=torch.bfloat16, device="cuda")
    tmap = torch.empty((S,), dtype=torch.int32, device="cuda")
    dw = torch.empty((S,), dtype=torch.float32, device="cuda")
    with torch.cuda.device(0):
        st = lib.ds_moe_dispatch_noalloc(x.data_ptr(), idx.data_ptr(), w.data_ptr(),
                                         offsets.data_ptr(), disp.data_ptr(), tmap.data_ptr(),
                                         dw.data_ptr(), 64, H, E, K, other.cuda_stream)
    assert st == ds_kernels.DS_ERR_UNSUPPORTED
    assert "stream" in lib.ds_last_error().decode()
