"""GPU parity of the tcgen05 grouped GEMMs (moe_gemm1, moe_gemm1_swiglu, moe_gemm2) and the
MLA kv up-projection against the f32 CPU oracle, through the C ABI.  Mirrors
tests/test_moe_gemm1.py, tests/test_moe_gemm2.py and tests/test_kv_upproj.py of the
reference (same input distributions and round-robin expert counts), plus skewed and empty
expert groups.

Tolerances: |out - ref| <= 5e-2 + 2^-8 |ref| (the reference tests' atol for these GEMMs
plus the bf16 relative half-ulp of the output) and rel-L2 <= 1e-2 against the f32 oracle.
"""
import pytest
import torch

import oracle
from conftest import assert_bf16_close

pytestmark = pytest.mark.gpu

H, I, E, K = 2048, 1408, 64, 6


def ds():
    import ds_kernels
    return ds_kernels


def rel_l2(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return (torch.linalg.vector_norm(a - b) / torch.linalg.vector_norm(b).clamp_min(1e-30)).item()


def round_robin_offsets(S, E_=E):
    counts = torch.tensor([(S // E_) + (1 if e < S % E_ else 0) for e in range(E_)], dtype=torch.int32)
    return oracle.expert_offsets(counts)


def skewed_offsets(S, E_=E):
    # expert 0 empty, expert 1 gets most rows, a few singletons, the rest empty
    counts = torch.zeros(E_, dtype=torch.int32)
    rest = S
    for e in (5, 9, 33, 63):
        if rest > 0:
            counts[e] = 1
            rest -= 1
    counts[1] = rest
    return oracle.expert_offsets(counts)


_W1 = {}


def gemm1_state(S, seed=42):
    g = torch.Generator().manual_seed(seed)
    a = (torch.rand(S, H, generator=g) * 2 - 1).to(torch.bfloat16)
    if "w1" not in _W1:
        gw = torch.Generator().manual_seed(1234)
        _W1["w1"] = (torch.rand(E, 2 * I, H, generator=gw) * 0.1).to(torch.bfloat16)
    return a, _W1["w1"]


def _check(out, ref, atol=5e-2):
    assert_bf16_close(out, ref, atol)


@pytest.mark.parametrize("tokens", [1, 8, 32, 128])
def test_gemm1_round_robin(tokens):
    S = tokens * K
    a, w1 = gemm1_state(S)
    off = round_robin_offsets(S)
    w1d = w1.cuda()
    out = ds().moe_gemm1(a.cuda(), w1d, off.cuda())
    assert out.shape == (S, 2 * I) and out.dtype == torch.bfloat16
    ref = oracle.grouped_linear(a, w1, off)
    _check(out, ref)


@pytest.mark.parametrize("S", [300, 2000])
def test_gemm1_skewed_and_swiglu(S):
    a, w1 = gemm1_state(S, seed=S)
    off = skewed_offsets(S)
    w1d = w1.cuda()
    out = ds().moe_gemm1(a.cuda(), w1d, off.cuda())
    ref = oracle.grouped_linear(a, w1, off)
    _check(out, ref)
    fused = ds().moe_gemm1_swiglu(a.cuda(), w1d, off.cuda())
    assert fused.shape == (S, I)
    _check(fused, oracle.swiglu(ref), atol=5e-2)


def test_gemm1_uncovered_rows_are_zero():
    S = 200
    a, w1 = gemm1_state(S)
    counts = torch.zeros(E, dtype=torch.int32)
    counts[3] = 150  # rows 150..199 belong to no expert
    off = oracle.expert_offsets(counts)
    out = ds().moe_gemm1(a.cuda(), w1.cuda(), off.cuda())
    assert torch.all(out[150:] == 0)
    _check(out, oracle.grouped_linear(a, w1, off))


def test_gemm1_empty():
    w1 = torch.zeros(E, 2 * I, H, dtype=torch.bfloat16).cuda()
    out = ds().moe_gemm1(torch.empty(0, H, dtype=torch.bfloat16).cuda(), w1,
                         torch.zeros(E + 1, dtype=torch.int32).cuda())
    assert out.shape == (0, 2 * I)


_W2 = {}


@pytest.mark.parametrize("tokens,skew", [(1, False), (8, False), (32, False), (128, False),
                                         (400, True)])
def test_gemm2(tokens, skew):
    S = tokens * K
    g = torch.Generator().manual_seed(tokens)
    a = (torch.rand(S, I, generator=g) * 2 - 1).to(torch.bfloat16)
    if "w2" not in _W2:
        gw = torch.Generator().manual_seed(99)
        _W2["w2"] = (torch.rand(E, H, I, generator=gw) * 0.1).to(torch.bfloat16)
    w2 = _W2["w2"]
    off = skewed_offsets(S) if skew else round_robin_offsets(S)
    out = ds().moe_gemm2(a.cuda(), w2.cuda(), off.cuda())
    assert out.shape == (S, H)
    _check(out, oracle.grouped_linear(a, w2, off))


def test_gemm2_empty():
    out = ds().moe_gemm2(torch.empty(0, I, dtype=torch.bfloat16).cuda(),
                         torch.zeros(E, H, I, dtype=torch.bfloat16).cuda(),
                         torch.zeros(E + 1, dtype=torch.int32).cuda())
    assert out.shape == (0, H)


@pytest.mark.parametrize("rows", [1, 16, 64, 129, 4096])
def test_kv_upproj(rows):
    g = torch.Generator().manual_seed(rows)
    x = (torch.randn(rows, 512, generator=g) * 0.1).to(torch.bfloat16)
    w = (torch.randn(4096, 512, generator=g) * 0.02).to(torch.bfloat16)
    out = ds().kv_upproj(x.cuda(), w.cuda())
    assert out.shape == (rows, 4096)
    _check(out, oracle.kv_upproj(x, w))


def test_kv_upproj_3d():
    g = torch.Generator().manual_seed(5)
    x = (torch.randn(2, 32, 512, generator=g) * 0.1).to(torch.bfloat16)
    w = (torch.randn(4096, 512, generator=g) * 0.02).to(torch.bfloat16)
    out = ds().kv_upproj(x.cuda(), w.cuda())
    assert out.shape == (2, 32, 4096)
    _check(out.view(-1, 4096), oracle.kv_upproj(x.view(-1, 512), w))
