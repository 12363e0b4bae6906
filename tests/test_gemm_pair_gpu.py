"""CTA-pair tiling of the tcgen05 grouped GEMM (2-CTA clusters, cta_group::2 MMAs on 256 x 256
tiles) against single-CTA 128 x 256 tiles and the f32 oracle.

Both tilings sum every output element over the same k-blocks in the same order, so the pair
mode must reproduce the single-CTA result bit for bit; the oracle bound of the GEMM tests
(|out - ref| <= 5e-2 + 2^-8 |ref|) is checked as well.  Cases: ragged and skewed expert
groups (groups of 1 row, empty groups, a group that is not a multiple of 256 rows), the
SwiGLU and plain epilogues, a partial last n-tile, output rows through a row map, dense
problems, and the full config-2 layer.
"""
import pytest
import torch

import oracle
from conftest import assert_bf16_close

pytestmark = pytest.mark.gpu

H, I, E = 2048, 1408, 64


def ds():
    import ds_kernels
    return ds_kernels


class pair_mode:
    def __init__(self, mode):
        self.mode = mode

    def __enter__(self):
        self.prev = ds().gemm_pair_mode(self.mode)

    def __exit__(self, *exc):
        ds().gemm_pair_mode(self.prev)


def both(fn):
    """fn() under single-CTA tiles and under forced CTA pairs."""
    with pair_mode(0):
        a = fn()
    with pair_mode(1):
        b = fn()
    torch.cuda.synchronize()
    return a, b


def offsets_of(counts):
    return oracle.expert_offsets(torch.tensor(counts, dtype=torch.int32))


def counts_ragged(S, seed):
    g = torch.Generator().manual_seed(seed)
    c = torch.randint(0, 2 * S // E + 1, (E,), generator=g)
    c[3] = 0
    c[7] = 1
    c[11] = 257
    c[12] = 255
    c[13] = 256
    return c.tolist()


def test_pair_mode_switch():
    prev = ds().gemm_pair_mode(None)
    assert prev in (-1, 0, 1)
    with pair_mode(1):
        assert ds().gemm_pair_mode(None) == 1
    assert ds().gemm_pair_mode(None) == prev


@pytest.mark.parametrize("swiglu", [False, True])
@pytest.mark.parametrize("seed", [1, 2])
def test_gemm1_pair_bit_exact(swiglu, seed):
    counts = counts_ragged(3000, seed)
    off = offsets_of(counts)
    S = int(off[-1])
    g = torch.Generator().manual_seed(seed)
    a = (torch.rand(S, H, generator=g) * 2 - 1).to(torch.bfloat16)
    w1 = (torch.randn(E, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16)
    ad, wd, od = a.cuda(), w1.cuda(), off.cuda()
    fn = (lambda: ds().moe_gemm1_swiglu(ad, wd, od)) if swiglu else (lambda: ds().moe_gemm1(ad, wd, od))
    o1, o2 = both(fn)
    assert torch.equal(o1, o2)
    ref = oracle.grouped_linear(a, w1, off)
    if swiglu:
        ref = oracle.swiglu(ref)
    assert_bf16_close(o2, ref, 5e-2)


@pytest.mark.parametrize("counts", ["skewed", "ragged"])
def test_gemm2_pair_bit_exact(counts):
    if counts == "skewed":
        c = [0] * E
        c[1], c[5], c[9], c[63] = 1990, 1, 1, 8
    else:
        c = counts_ragged(2500, 7)
    off = offsets_of(c)
    S = int(off[-1])
    g = torch.Generator().manual_seed(3)
    h = torch.randn(S, I, generator=g).to(torch.bfloat16)
    w2 = (torch.randn(E, H, I, generator=g) * 0.02).to(torch.bfloat16)
    hd, wd, od = h.cuda(), w2.cuda(), off.cuda()
    o1, o2 = both(lambda: ds().moe_gemm2(hd, wd, od))
    assert torch.equal(o1, o2)
    assert_bf16_close(o2, oracle.grouped_linear(h, w2, off), 5e-2)


@pytest.mark.parametrize("I_", [1360, 10944 // 2 + 8])
def test_gemm1_pair_partial_last_n_tile(I_):
    # 2I not a multiple of 256: the last n-tile holds fewer than 128 valid columns per half
    G = 3
    off = offsets_of([700, 0, 513])
    S = int(off[-1])
    g = torch.Generator().manual_seed(I_)
    a = torch.randn(S, 512, generator=g).to(torch.bfloat16)
    w1 = (torch.randn(G, 2 * I_, 512, generator=g) * 0.05).to(torch.bfloat16)
    ad, wd, od = a.cuda(), w1.cuda(), off.cuda()
    o1, o2 = both(lambda: ds().moe_gemm1_swiglu(ad, wd, od))
    assert torch.equal(o1, o2)
    ref = oracle.swiglu(oracle.grouped_linear(a, w1, off))
    assert_bf16_close(o2, ref, 5e-2)


@pytest.mark.parametrize("rows,out_dim", [(777, 4096), (16384, 4096), (1000, 4096 + 72)])
def test_kv_upproj_pair_bit_exact(rows, out_dim):
    g = torch.Generator().manual_seed(rows)
    x = torch.randn(rows, 512, generator=g).to(torch.bfloat16)
    w = (torch.randn(out_dim, 512, generator=g) * 0.05).to(torch.bfloat16)
    xd, wd = x.cuda(), w.cuda()
    o1, o2 = both(lambda: ds().kv_upproj(xd, wd))
    assert torch.equal(o1, o2)
    ref = x.float() @ w.float().t()
    assert_bf16_close(o2, ref, 5e-2)


def test_expert_mlp_row_map_pair_bit_exact():
    # output rows scattered through a row map (the mapped copy-out epilogue)
    c = counts_ragged(2000, 11)[:8]
    off = offsets_of(c)
    R = int(off[-1])
    G = len(c)
    g = torch.Generator().manual_seed(5)
    rows = torch.randn(R, H, generator=g).to(torch.bfloat16)
    w1 = (torch.randn(G, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(G, H, I, generator=g) * 0.02).to(torch.bfloat16)
    perm = torch.randperm(R, generator=g).to(torch.int32)
    rd, od, w1d, w2d, pd = rows.cuda(), off.cuda(), w1.cuda(), w2.cuda(), perm.cuda()

    def run():
        out = torch.zeros(R, H, dtype=torch.bfloat16, device="cuda")
        return ds().moe_expert_mlp(rd, od, w1d, w2d, out=out, out_row_map=pd)

    o1, o2 = both(run)
    assert torch.equal(o1, o2)


def test_fused_layer_cfg2_pair_bit_exact():
    # the config-2 layer (T = 8192): routed GEMMs over 64 ragged groups plus the shared expert
    from moe_fused import FusedMoELayer
    import synthetic
    dev = torch.device("cuda", 0)
    Wd = synthetic.make_layer_weights(0, dev, H, I, E, 2)
    layer = FusedMoELayer.from_packed(Wd.gate, Wd.packed_w1, Wd.w2, Wd.shared_w1, Wd.shared_w2,
                                      top_k=6)
    g = torch.Generator(device=dev).manual_seed(2)
    x = torch.randn(8192, H, generator=g, device=dev).to(torch.bfloat16)
    o1, o2 = both(lambda: layer(x).clone())
    assert torch.equal(o1, o2)
