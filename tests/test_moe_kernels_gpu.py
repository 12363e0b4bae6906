"""GPU parity of the MoE routing / scan / dispatch / combine / SwiGLU kernels against the CPU
oracle, through the C ABI (ds_kernels).  Mirrors tests/test_moe_routing_kernel.py,
tests/test_moe_scan_kernel.py, tests/test_moe_dispatch_kernel.py,
tests/test_moe_combine_kernel.py and tests/test_swiglu_kernel.py of the reference, with
bit-exact checks where the reference only compared sets.

Tolerances: integer outputs bit-exact; routing weights atol 1e-6 (f32 softmax, 1 ulp of
exp/divide); bf16 outputs |out - ref| <= atol + 2^-8 |ref| (atol = the reference test's:
2e-2 single-slot combine, 5e-2 multi-slot combine, 1e-2 swiglu; 2^-8 = bf16 relative
half-ulp) and rel-L2 <= 1e-2 against the f32 oracle.
"""
import os

import pytest
import torch

import oracle
from conftest import assert_bf16_close

pytestmark = pytest.mark.gpu

E, K, H = 64, 6, 2048
ROUTE_T = [1, 3, 32, 63, 64, 65, 128, 1000]


def rel_l2(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return (torch.linalg.vector_norm(a - b) / torch.linalg.vector_norm(b).clamp_min(1e-30)).item()


def ds():
    import ds_kernels
    return ds_kernels


# ------------------------------------------------------------------------------ routing
@pytest.mark.parametrize("T", ROUTE_T)
def test_routing_bit_exact(T):
    g = torch.Generator().manual_seed(100 + T)
    logits = torch.randn(T, E, generator=g)
    idx, w, counts = ds().moe_routing(logits.cuda(), top_k=K)
    ridx, rw = oracle.route(logits, K)
    assert idx.shape == (T, K) and w.shape == (T, K) and counts.shape == (E,)
    assert torch.equal(idx.cpu(), ridx)
    torch.testing.assert_close(w.cpu(), rw, atol=1e-6, rtol=0)
    assert torch.equal(counts.cpu(), oracle.expert_counts(ridx, E))
    assert int(counts.sum()) == T * K


def test_routing_ties_lower_index():
    logits = torch.zeros(16, E)
    idx, w, counts = ds().moe_routing(logits.cuda(), top_k=K)
    assert torch.equal(idx.cpu(), torch.arange(K, dtype=torch.int32).expand(16, K))
    for t in range(16):
        assert len(set(idx[t].tolist())) == K
    assert int(counts.sum()) == 16 * K


def test_routing_partial_ties_and_small_E():
    g = torch.Generator().manual_seed(5)
    logits = torch.randint(-2, 3, (257, 24), generator=g).float()  # many exact ties
    for k in (1, 2, 6, 8):
        idx, w, counts = ds().moe_routing(logits.cuda(), top_k=k)
        ridx, rw = oracle.route(logits, k)
        assert torch.equal(idx.cpu(), ridx), k
        torch.testing.assert_close(w.cpu(), rw, atol=1e-6, rtol=0)
        assert torch.equal(counts.cpu(), oracle.expert_counts(ridx, 24))


def test_routing_cfg1_zipf_full_size():
    T = 16384
    logits = oracle.zipf_logits(T, E, seed=11)
    idx, w, counts = ds().moe_routing(logits.cuda(), top_k=K)
    ridx, rw = oracle.route(logits, K)
    assert torch.equal(idx.cpu(), ridx)
    torch.testing.assert_close(w.cpu(), rw, atol=1e-6, rtol=0)
    assert torch.equal(counts.cpu(), oracle.expert_counts(ridx, E))
    assert int(counts.max()) > T // 2  # the Zipf bias concentrates load


def test_routing_rejects_bad_args():
    with pytest.raises(RuntimeError):
        ds().moe_routing(torch.randn(4, 65).cuda(), top_k=6)
    with pytest.raises(RuntimeError):
        ds().moe_routing(torch.randn(4, 64, dtype=torch.float64).cuda(), top_k=6)
    with pytest.raises(RuntimeError):
        ds().moe_routing(torch.randn(4, 64), top_k=6)


# ------------------------------------------------------------------------------ scan
def test_scan_known_answers(golden_dir):
    ka = torch.load(os.path.join(golden_dir, "known_answers.pt"), weights_only=False)
    for key in ("scan_random", "scan_zeros", "scan_single", "scan_uniform", "scan_skewed",
                "scan_sentinel"):
        counts, offsets = ka[key]
        out = ds().moe_scan(counts.to(torch.int32).cuda())
        assert torch.equal(out.cpu(), offsets.to(torch.int32)), key


def test_scan_large_and_random():
    g = torch.Generator().manual_seed(3)
    for n in (2, 63, 64, 65, 1000, 1024, 1025, 5000, 16383, 16384, 16385, 40000):
        c = torch.randint(0, 1000, (n,), generator=g, dtype=torch.int32)
        out = ds().moe_scan(c.cuda())
        assert torch.equal(out.cpu(), oracle.expert_offsets(c)), n


# ------------------------------------------------------------------------------ dispatch
def _pipeline(T, logits=None, seed=42):
    g = torch.Generator().manual_seed(seed)
    if logits is None:
        logits = torch.randn(T, E, generator=g)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    idx, w, counts = ds().moe_routing(logits.cuda(), top_k=K)
    offsets = ds().moe_scan(counts)
    disp, tmap, dw = ds().moe_dispatch(x.cuda(), idx, w, offsets)
    return logits, x, idx, w, counts, offsets, disp, tmap, dw


@pytest.mark.parametrize("T", [1, 32, 65, 128, 1000])
def test_dispatch_bit_exact(T):
    logits, x, idx, w, counts, offsets, disp, tmap, dw = _pipeline(T)
    ridx, rw = oracle.route(logits, K)
    rdisp, rtmap, rdw, _, roff = oracle.dispatch(x, ridx, rw, E)
    assert torch.equal(offsets.cpu(), roff)
    assert torch.equal(tmap.cpu(), rtmap)
    assert torch.equal(disp.cpu(), rdisp)
    # weights are copied, not recomputed: exact against the kernel's own routing weights
    rdw_k = w.cpu().reshape(-1)[torch.sort(idx.cpu().reshape(-1).long(), stable=True).indices]
    assert torch.equal(dw.cpu(), rdw_k)
    # each token appears exactly K times (tests/test_moe_dispatch_kernel.py:114-133)
    assert torch.all(torch.bincount(tmap.cpu().long(), minlength=T) == K)


def test_dispatch_cfg1_full_size():
    T = 16384
    logits = oracle.zipf_logits(T, E, seed=12)
    logits, x, idx, w, counts, offsets, disp, tmap, dw = _pipeline(T, logits=logits)
    ridx, rw = oracle.route(logits, K)
    # permutation and offsets bit-exact; rows checked against a device gather by token_map
    flat_e = ridx.reshape(-1).long()
    perm = torch.sort(flat_e, stable=True).indices
    rtmap = torch.arange(T).repeat_interleave(K)[perm].to(torch.int32)
    assert torch.equal(tmap.cpu(), rtmap)
    assert torch.equal(offsets.cpu(), oracle.expert_offsets(oracle.expert_counts(ridx, E)))
    gathered = x.cuda()[tmap.long()]
    assert torch.equal(disp, gathered)


def test_dispatch_empty():
    x = torch.empty(0, H, dtype=torch.bfloat16).cuda()
    idx = torch.empty(0, K, dtype=torch.int32).cuda()
    w = torch.empty(0, K).cuda()
    off = torch.zeros(E + 1, dtype=torch.int32).cuda()
    d, tm, dw = ds().moe_dispatch(x, idx, w, off)
    assert d.shape == (0, H) and tm.shape == (0,) and dw.shape == (0,)


# ------------------------------------------------------------------------------ combine
def _check_combine(eo, tm, dw, T, atol):
    out = ds().moe_combine(eo.cuda(), tm.cuda(), dw.cuda(), T)
    ref = oracle.combine(eo, tm, dw, T)
    assert out.shape == (T, eo.shape[1]) and out.dtype == torch.bfloat16
    assert_bf16_close(out, ref, atol)
    return out


@pytest.mark.parametrize("T", [1, 32, 128])
def test_combine_single_slot(T):
    g = torch.Generator().manual_seed(0)
    eo = torch.randn(T, H, generator=g).to(torch.bfloat16)
    _check_combine(eo, torch.arange(T, dtype=torch.int32), torch.rand(T, generator=g), T, 2e-2)


@pytest.mark.parametrize("T", [1, 32, 128])
def test_combine_multi_slot(T):
    g = torch.Generator().manual_seed(1)
    eo = torch.randn(T * K, H, generator=g).to(torch.bfloat16)
    tm = torch.repeat_interleave(torch.arange(T, dtype=torch.int32), K)
    _check_combine(eo, tm, torch.rand(T * K, generator=g), T, 5e-2)


@pytest.mark.parametrize("T", [1, 32, 128])
def test_combine_arbitrary_multiplicity(T):
    g = torch.Generator().manual_seed(2)
    S = T * K
    eo = torch.randn(S, H, generator=g).to(torch.bfloat16)
    tm = torch.randint(0, T, (S,), generator=g, dtype=torch.int32)
    _check_combine(eo, tm, torch.rand(S, generator=g), T, 5e-2)


def test_combine_heavy_token_and_empty_tokens():
    g = torch.Generator().manual_seed(4)
    T, S = 50, 300
    eo = torch.randn(S, H, generator=g).to(torch.bfloat16)
    tm = torch.full((S,), 7, dtype=torch.int32)  # one token receives 300 slots (> 32)
    tm[::10] = 3
    dw = torch.rand(S, generator=g) / 50
    _check_combine(eo, tm, dw, T, 2e-2)


def test_combine_many_long_segments():
    # every token has 9-40 slots: all of them go through the overflow list to the batched
    # long-segment kernel
    g = torch.Generator().manual_seed(7)
    T, S = 300, 7000
    eo = torch.randn(S, H, generator=g).to(torch.bfloat16)
    tm = torch.randint(0, T, (S,), generator=g, dtype=torch.int32)
    dw = torch.rand(S, generator=g) / 20
    _check_combine(eo, tm, dw, T, 2e-2)


def test_combine_more_tokens_than_one_scan_tile():
    # T > 16384: the single-CTA scan of the per-token counts carries over several tiles
    g = torch.Generator().manual_seed(8)
    T = 20000
    S = T + 3000
    eo = torch.randn(S, H, generator=g).to(torch.bfloat16)
    tm = torch.cat([torch.arange(T, dtype=torch.int32),
                    torch.randint(0, T, (S - T,), generator=g, dtype=torch.int32)])
    _check_combine(eo, tm, torch.rand(S, generator=g), T, 2e-2)


def test_combine_known_answer(golden_dir):
    c = torch.load(os.path.join(golden_dir, "known_answers.pt"), weights_only=False)["combine"]
    # H=64 in the fixture
    out = ds().moe_combine(c["eo"].cuda(), c["token_map"].cuda(), c["dw"].cuda(), c["T"])
    assert_bf16_close(out, c["out"], 2e-2)


@pytest.mark.parametrize("T", [1, 32, 128])
def test_combine_zero_weights_exact_zero(T):
    g = torch.Generator().manual_seed(5)
    S = T * K
    eo = torch.randn(S, H, generator=g).to(torch.bfloat16).cuda()
    tm = torch.randint(0, T, (S,), generator=g, dtype=torch.int32).cuda()
    out = ds().moe_combine(eo, tm, torch.zeros(S).cuda(), T)
    assert torch.all(out == 0)


def test_combine_deterministic():
    g = torch.Generator().manual_seed(6)
    T, S = 700, 4200
    eo = torch.randn(S, H, generator=g).to(torch.bfloat16).cuda()
    tm = torch.randint(0, T, (S,), generator=g, dtype=torch.int32).cuda()
    dw = torch.rand(S, generator=g).cuda()
    a = ds().moe_combine(eo, tm, dw, T)
    b = ds().moe_combine(eo, tm, dw, T)
    assert torch.equal(a, b)


@pytest.mark.parametrize("T", [1, 32, 128])
def test_route_dispatch_combine_end_to_end(T):
    # tests/test_moe_combine_kernel.py:166-214: combining the dispatched inputs reproduces
    # sum_k w_k * x_t
    logits, x, idx, w, counts, offsets, disp, tmap, dw = _pipeline(T, seed=7)
    out = ds().moe_combine(disp, tmap, dw, T)
    ref = x.float() * w.cpu().sum(1, keepdim=True)
    assert_bf16_close(out, ref, 2e-2)


# ------------------------------------------------------------------------------ swiglu
@pytest.mark.parametrize("rows", [1, 8, 32, 128, 256, 4099])
def test_swiglu(rows):
    g = torch.Generator().manual_seed(rows)
    x = (torch.rand(rows, 2 * 1408, generator=g) * 4 - 2).to(torch.bfloat16)
    out = ds().swiglu(x.cuda())
    ref = oracle.swiglu(x)
    assert out.shape == (rows, 1408)
    assert_bf16_close(out, ref, 1e-2)


@pytest.mark.parametrize("rows", [1, 256, 4099])
def test_swiglu_equals_the_bf16_torch_expression(rows):
    # The drop-in rounds silu(gate) to bf16 before the product, as F.silu(gate) * up does on
    # bf16 tensors (the reference model's expert, src/reference/moe.py:19, and its swiglu
    # test's oracle, tests/test_swiglu_kernel.py): bit for bit.
    import torch.nn.functional as F
    g = torch.Generator().manual_seed(rows)
    x = (torch.rand(rows, 2 * 1408, generator=g) * 4 - 2).to(torch.bfloat16).cuda()
    out = ds().swiglu(x)
    ref = F.silu(x[:, :1408]) * x[:, 1408:]
    assert torch.equal(out, ref)


def test_swiglu_odd_width_and_empty():
    x = (torch.rand(5, 2 * 6) * 4 - 2).to(torch.bfloat16)
    out = ds().swiglu(x.cuda())
    assert_bf16_close(out, oracle.swiglu(x), 1e-2)
    e = ds().swiglu(torch.empty(0, 2816, dtype=torch.bfloat16).cuda())
    assert e.shape == (0, 1408)
