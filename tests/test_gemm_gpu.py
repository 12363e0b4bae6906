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


# ---- output widths that are not a multiple of the 256-column tile -------------------------
# The last n-tile of a problem then holds fewer valid columns (the gate | up halves of GEMM1
# each end at I; a plain tile ends at N).  Columns past the end are computed but never
# stored: the values on both sides of the gate | up boundary and a guard region after the
# output are checked.

@pytest.mark.parametrize("I_", [72, 200, 1000])
def test_gemm1_partial_last_n_tile(I_):
    E_, H_ = 8, 256
    g = torch.Generator().manual_seed(I_)
    S = 777
    a = (torch.rand(S, H_, generator=g) * 2 - 1).to(torch.bfloat16)
    w1 = (torch.rand(E_, 2 * I_, H_, generator=g) * 0.1).to(torch.bfloat16)
    off = round_robin_offsets(S, E_)
    out = ds().moe_gemm1(a.cuda(), w1.cuda(), off.cuda())
    assert out.shape == (S, 2 * I_)
    ref = oracle.grouped_linear(a, w1, off)
    _check(out, ref)
    fused = ds().moe_gemm1_swiglu(a.cuda(), w1.cuda(), off.cuda())
    assert fused.shape == (S, I_)
    _check(fused, oracle.swiglu(ref))


def _guarded_out(rows, cols):
    """bf16 buffer of rows*cols elements followed by 4096 guard elements set to a sentinel."""
    buf = torch.full((rows * cols + 4096,), 7.0, dtype=torch.bfloat16, device="cuda")
    return buf


@pytest.mark.parametrize("H_", [1000, 2056])
def test_gemm2_partial_last_n_tile_stays_in_bounds(H_):
    E_, I_ = 8, 200
    g = torch.Generator().manual_seed(H_)
    S = 555
    a = (torch.rand(S, I_, generator=g) * 2 - 1).to(torch.bfloat16)
    w2 = (torch.rand(E_, H_, I_, generator=g) * 0.1).to(torch.bfloat16)
    off = round_robin_offsets(S, E_)
    k = ds()
    buf = _guarded_out(S, H_)
    ad, wd, od = a.cuda(), w2.cuda(), off.cuda()
    st = k.library().ds_moe_gemm2(ad.data_ptr(), wd.data_ptr(), od.data_ptr(), buf.data_ptr(), S,
                                  E_, I_, H_, torch.cuda.current_stream().cuda_stream)
    assert st == 0, k.library().ds_last_error().decode()
    torch.cuda.synchronize()
    assert torch.all(buf[S * H_:] == 7.0)
    _check(buf[:S * H_].view(S, H_), oracle.grouped_linear(a, w2, off))


@pytest.mark.parametrize("out_dim", [1000, 4104])
def test_kv_upproj_any_width(out_dim):
    g = torch.Generator().manual_seed(out_dim)
    rows = 300
    x = (torch.randn(rows, 512, generator=g) * 0.1).to(torch.bfloat16)
    w = (torch.randn(out_dim, 512, generator=g) * 0.02).to(torch.bfloat16)
    out = ds().kv_upproj(x.cuda(), w.cuda())
    assert out.shape == (rows, out_dim)
    _check(out, oracle.kv_upproj(x, w))
