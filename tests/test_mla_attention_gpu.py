"""MLA attention on the tcgen05 kernels against the f32 CPU oracle.

* The attention core (ds_mla_attention: S = Q K^T and O += P V on the tensor cores with the
  online softmax between them) against oracle.mla_attention (src/reference/mla.py:355-378)
  at sequence lengths that are and are not multiples of the 128-row tiles.
* The whole MLA forward (ds_mla_forward / mla.FusedMLA: fused q|kv_a projection, latent
  RMSNorm, kv_b projection, RoPE, attention, o_proj) against oracle.mla_forward — itself pinned
  to the reference's DeepSeekMLA by tests/test_oracle_golden.py — on the golden fixtures'
  weights (YaRN factor 40 and plain RoPE), and at the full config-3 size (batch 4, seq 4096,
  hidden 2048, 16 heads, plain RoPE theta 10000) on a sample of rows of every sequence.
The oracle computes in f32 from the bf16-rounded inputs and weights; the bound is the
BASELINE float contract, max-abs <= 2e-2 and rel-L2 <= 1e-2.
"""
import math
import os

import pytest
import torch

import oracle
from conftest import GOLDEN

pytestmark = pytest.mark.gpu


def check(out, ref, atol=2e-2, rel=1e-2):
    o = out.float().cpu()
    r = ref.float().cpu()
    d = (o - r).abs().max().item()
    e = ((o - r).norm() / r.norm()).item()
    assert d <= atol and e <= rel, (d, e)


def _attention_inputs(B, S, heads, seed):
    g = torch.Generator().manual_seed(seed)
    ldq = heads * 192 + 576
    qkv = torch.randn(B * S, ldq, generator=g).to(torch.bfloat16)
    kv = torch.randn(B * S, heads * 256, generator=g).to(torch.bfloat16)
    return qkv, kv


def _oracle_attention(qkv, kv, B, S, heads, scale):
    q = qkv[:, :heads * 192].float().view(B, S, heads, 192).transpose(1, 2)
    kr = qkv[:, heads * 192 + 512:].float().view(B, S, 1, 64).transpose(1, 2)
    kvf = kv.float().view(B, S, heads, 256).transpose(1, 2)
    k = torch.cat([kvf[..., :128], kr.expand(B, heads, S, 64)], dim=-1)
    v = kvf[..., 128:]
    o = oracle.mla_attention(q, k, v, scale)
    return o.transpose(1, 2).reshape(B * S, heads * 128)


@pytest.mark.parametrize("B,S,heads", [(1, 8, 1), (1, 128, 1), (2, 200, 3), (1, 1024, 2),
                                       (3, 520, 16)])
def test_attention_core(B, S, heads):
    import ds_kernels
    qkv, kv = _attention_inputs(B, S, heads, seed=S + heads)
    scale = 192 ** -0.5
    out = ds_kernels.mla_attention(qkv.cuda(), kv.cuda(), B, S, heads, scale)
    assert out.shape == (B * S, heads * 128)
    check(out, _oracle_attention(qkv, kv, B, S, heads, scale))
    assert ds_kernels.device_status() == ds_kernels.DS_OK


def test_attention_core_peaked_scores():
    # a large softmax scale makes every row's maximum move between kv blocks many times
    import ds_kernels
    B, S, heads = 1, 640, 2
    qkv, kv = _attention_inputs(B, S, heads, seed=11)
    scale = 0.5
    out = ds_kernels.mla_attention(qkv.cuda(), kv.cuda(), B, S, heads, scale)
    check(out, _oracle_attention(qkv, kv, B, S, heads, scale))


def _fixture_module(name):
    from oracle.modules import OracleMLA
    fx = torch.load(os.path.join(GOLDEN, name))
    bf = lambda t: t.to(torch.bfloat16).float()  # noqa: E731  (the bf16-rounded operands)
    mod = OracleMLA(bf(fx["w_q"]), bf(fx["w_kva"]), fx["norm_w"], bf(fx["w_kvb"]), bf(fx["w_o"]),
                    bf(fx["cos"]), bf(fx["sin"]), fx["softmax_scale"], fx["heads"])
    return fx, mod


@pytest.mark.parametrize("name", ["mla_forward_yarn40.pt", "mla_forward_plain.pt"])
def test_fused_mla_on_the_reference_fixture_weights(name):
    from mla import FusedMLA
    fx, mod = _fixture_module(name)
    fused = FusedMLA(mod, device=torch.device("cuda"))
    x = fx["x"].to(torch.bfloat16)
    out = fused(x.cuda())
    assert out.shape == x.shape and out.dtype == torch.bfloat16
    ref = mod(x.float())
    check(out, ref)
    # the reference module's own f32 output, for scale: the bf16 path stays within 5e-2
    assert (out.float().cpu() - fx["out"]).abs().max().item() < 5e-2


def test_fused_mla_position_ids():
    # explicit position_ids equal to the default give the same bits; positions shifted by 5
    # rotate with table rows 5.. and match the oracle run on the shifted tables
    from mla import FusedMLA
    from oracle.modules import OracleMLA
    fx = torch.load(os.path.join(GOLDEN, "mla_forward_plain.pt"))
    bf = lambda t: t.to(torch.bfloat16).float()  # noqa: E731
    cos, sin = oracle.yarn_cos_sin(64, scaling_factor=1.0)
    mod = OracleMLA(bf(fx["w_q"]), bf(fx["w_kva"]), fx["norm_w"], bf(fx["w_kvb"]), bf(fx["w_o"]),
                    bf(cos), bf(sin), fx["softmax_scale"], fx["heads"])
    fused = FusedMLA(mod, device=torch.device("cuda"))
    x = fx["x"].to(torch.bfloat16)
    S = x.shape[1]
    a = fused(x.cuda())
    b = fused(x.cuda(), position_ids=torch.arange(S, device="cuda")[None])
    assert torch.equal(a, b)
    c = fused(x.cuda(), position_ids=torch.arange(S, device="cuda")[None] + 5)
    ref = oracle.mla_forward(x.float(), mod.q_proj.weight, mod.kv_a_proj_with_mqa.weight,
                             mod.kv_a_layernorm.weight, mod.kv_b_proj.weight, mod.o_proj.weight,
                             bf(cos)[5:], bf(sin)[5:], fx["softmax_scale"], fx["heads"])
    check(c, ref)


def test_mla_forward_config3_full_size():
    import ds_kernels
    B, S, Hd, heads = 4, 4096, 2048, 16
    g = torch.Generator().manual_seed(2)
    x = torch.randn(B, S, Hd, generator=g).to(torch.bfloat16)

    def w(*shape):
        return (torch.randn(*shape, generator=g) * 0.02).to(torch.bfloat16)

    w_q, w_kva = w(heads * 192, Hd), w(576, Hd)
    norm_w = torch.rand(512, generator=g) + 0.5
    w_kvb, w_o = w(heads * 256, 512), w(Hd, heads * 128)
    cos, sin = oracle.yarn_cos_sin(S, scaling_factor=1.0)
    cos, sin = cos.to(torch.bfloat16), sin.to(torch.bfloat16)
    scale = 192 ** -0.5
    out = ds_kernels.mla_forward(x.cuda(), torch.cat([w_q, w_kva]).cuda(), norm_w.cuda(),
                                 w_kvb.cuda(), w_o.cuda(), cos.cuda(), sin.cuda(), scale, heads)
    torch.cuda.synchronize()
    rows = torch.tensor([0, 1, 127, 128, 1000, 2047, 2048, 3001, 4094, 4095])
    ref = oracle.mla_forward_rows(x, w_q, w_kva, norm_w, w_kvb, w_o, cos, sin, scale, heads, rows)
    check(out[:, rows], ref)
    assert ds_kernels.device_status() == ds_kernels.DS_OK
