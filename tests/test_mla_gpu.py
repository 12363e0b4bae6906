"""GPU parity of the MLA projection bandwidth kernels (rms_norm, rope) against the f32 CPU
oracle, through the C ABI.  Mirrors tests/test_rms_norm.py and tests/test_rope_kernel.py of
the reference (atol 1e-2, plus the 2^-8 |ref| relative half-ulp of a bf16 output), including
their shapes, plus the BASELINE config-3 full size
(B=4, S=4096, 16 heads) and the committed golden tables."""
import os

import pytest
import torch

import oracle
from conftest import assert_bf16_close

pytestmark = pytest.mark.gpu


def ds():
    import ds_kernels
    return ds_kernels


def rel_l2(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return (torch.linalg.vector_norm(a - b) / torch.linalg.vector_norm(b).clamp_min(1e-30)).item()


@pytest.mark.parametrize("shape,scale,ones", [((4, 512), 0.5, True), ((8, 512), 0.5, True),
                                              ((16, 512), 0.3, False), ((2, 32, 512), 1.0, True),
                                              ((64, 512), 0.5, True), ((1000, 512), 1.0, False),
                                              ((7, 96), 1.0, False), ((5, 2048), 1.0, False)])
def test_rms_norm(shape, scale, ones):
    g = torch.Generator().manual_seed(sum(shape))
    x = (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16)
    H = shape[-1]
    w = torch.ones(H) if ones else torch.randn(H, generator=g).abs() + 0.5
    out = ds().rms_norm(x.cuda(), w.cuda(), 1e-6)
    assert out.shape == x.shape and out.dtype == torch.bfloat16
    ref = oracle.rms_norm(x, w, 1e-6)
    assert_bf16_close(out, ref, 1e-2)
    assert not torch.isnan(out).any() and not torch.isinf(out).any()


def test_rms_norm_odd_pairs_path():
    x = torch.randn(9, 34).to(torch.bfloat16)
    w = torch.rand(34) + 0.5
    out = ds().rms_norm(x.cuda(), w.cuda())
    assert_bf16_close(out, oracle.rms_norm(x, w), 1e-2)


def test_rms_norm_cfg3_full():
    g = torch.Generator().manual_seed(2)
    x = torch.randn(4 * 4096, 512, generator=g).to(torch.bfloat16)
    w = torch.rand(512, generator=g) + 0.5
    out = ds().rms_norm(x.cuda(), w.cuda())
    assert_bf16_close(out, oracle.rms_norm(x, w), 1e-2)


@pytest.mark.parametrize("rows,H", [(1, 2048), (7, 2048), (1000, 2048), (33, 512), (5, 96)])
def test_rms_norm_residual(rows, H):
    g = torch.Generator().manual_seed(rows + H)
    x = torch.randn(rows, H, generator=g).to(torch.bfloat16)
    r = (torch.randn(rows, H, generator=g) * 2).to(torch.bfloat16)
    w = torch.rand(H, generator=g) + 0.5
    n, s = ds().rms_norm_residual(x.cuda(), r.cuda(), w.cuda())
    rn, rs = oracle.rms_norm_residual(x, r, w)
    assert torch.equal(s.cpu(), rs)  # the residual sum is bit-exact
    assert_bf16_close(n, rn, 1e-2)


def _rope_inputs(bsz, seq, heads=16, seed=0, scaling=40.0):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(bsz, heads, seq, 64, generator=g) * 0.5).to(torch.bfloat16)
    k = (torch.randn(bsz, 1, seq, 64, generator=g) * 0.5).to(torch.bfloat16)
    cos, sin = oracle.yarn_cos_sin(seq, scaling_factor=scaling)
    pos = torch.arange(seq).unsqueeze(0).expand(bsz, -1)
    c = cos[pos].unsqueeze(1).to(torch.bfloat16)
    s = sin[pos].unsqueeze(1).to(torch.bfloat16)
    return q, k, c, s


@pytest.mark.parametrize("bsz,seq,heads,scaling", [(1, 16, 16, 40.0), (2, 64, 16, 40.0),
                                                   (1, 32, 16, 1.0), (3, 7, 4, 40.0),
                                                   (2, 100, 16, 40.0), (1, 20, 40, 1.0)])
def test_rope(bsz, seq, heads, scaling):
    q, k, c, s = _rope_inputs(bsz, seq, heads, seed=seq, scaling=scaling)
    qr, kr = ds().rope(q.cuda(), k.cuda(), c.cuda(), s.cuda())
    assert qr.shape == q.shape and kr.shape == k.shape and qr.dtype == torch.bfloat16
    rq, rk = oracle.rope(q, k, c, s)
    assert_bf16_close(qr, rq, 1e-2)
    assert_bf16_close(kr, rk, 1e-2)
    assert not torch.isnan(qr).any() and not torch.isinf(kr).any()


def test_rope_cfg3_full():
    q, k, c, s = _rope_inputs(4, 4096, 16, seed=2, scaling=1.0)
    qr, kr = ds().rope(q.cuda(), k.cuda(), c.cuda(), s.cuda())
    rq, rk = oracle.rope(q, k, c, s)
    assert_bf16_close(qr, rq, 1e-2)
    assert_bf16_close(kr, rk, 1e-2)


def test_rope_rms_against_golden(golden_dir):
    fx = torch.load(os.path.join(golden_dir, "mla_yarn40.pt"), weights_only=False)
    q, k = fx["q_pe"].to(torch.bfloat16), fx["k_pe"].to(torch.bfloat16)
    c = fx["cos"][None, None].expand(fx["bsz"], 1, -1, -1).contiguous().to(torch.bfloat16)
    s = fx["sin"][None, None].expand(fx["bsz"], 1, -1, -1).contiguous().to(torch.bfloat16)
    qr, kr = ds().rope(q.cuda(), k.cuda(), c.cuda(), s.cuda())
    # inputs and tables are rounded to bf16 before the kernel; the golden is f32 end to end
    assert_bf16_close(qr, fx["q_rot"], 3e-2)
    assert_bf16_close(kr, fx["k_rot"], 3e-2)
    x = fx["latent"].to(torch.bfloat16)
    out = ds().rms_norm(x.cuda(), fx["norm_weight"].cuda())
    assert_bf16_close(out, fx["normed"], 3e-2)
