"""MLA decode over the latent KV cache against the f32 CPU oracle.

* FusedMLA.prefill fills a LatentKVCache with a prompt's raw latents / k_pe while running the
  forward; FusedMLA.decode then runs one token per sequence (ds_mla_decode_step: absorbed
  query/output weights, split-KV tcgen05 attention over the cached latent, combine) and must
  match the oracle's forward row at the new position (oracle.mla_forward_rows on the whole
  token sequence so far) step after step.
* A config-4-shaped step (64 sequences, 2048 cached positions of N(0,1) latents / k_pe written
  through the reference's own update() API, hidden 2048, 16 heads) against
  oracle.mla_decode_step on a sample of sequences.
* Cache lengths around the 128-token chunks, and the first token of an empty cache.
Weights N(0, 0.02^2) as in the BASELINE configs; bound: the BASELINE float contract,
max-abs <= 2e-2 and rel-L2 <= 1e-2.
"""
import math

import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

HEADS = 16


def check(out, ref, atol=2e-2, rel=1e-2):
    o = out.float().cpu()
    r = ref.float().cpu()
    d = (o - r).abs().max().item()
    e = ((o - r).norm() / r.norm()).item()
    assert d <= atol and e <= rel, (d, e)


def _module(hidden, seed, max_pos, scaling=40.0, std=0.02):
    from oracle.modules import OracleMLA
    g = torch.Generator().manual_seed(seed)
    bf = lambda t: t.to(torch.bfloat16).float()  # noqa: E731

    def w(*shape):
        return bf(torch.randn(*shape, generator=g) * std)

    cos, sin = oracle.yarn_cos_sin(max_pos, scaling_factor=scaling)
    ms = 0.1 * 0.707 * math.log(scaling) + 1.0 if scaling > 1 else 1.0
    scale = 192 ** -0.5 * ms * ms
    return OracleMLA(w(HEADS * 192, hidden), w(576, hidden), torch.rand(512, generator=g) + 0.5,
                     w(HEADS * 256, 512), w(hidden, HEADS * 128), bf(cos), bf(sin), scale, HEADS)


def _rows(mod, x, rows):
    return oracle.mla_forward_rows(x, mod.q_proj.weight, mod.kv_a_proj_with_mqa.weight,
                                   mod.kv_a_layernorm.weight, mod.kv_b_proj.weight,
                                   mod.o_proj.weight, mod.rotary_emb.cos_cached,
                                   mod.rotary_emb.sin_cached, mod.softmax_scale, HEADS, rows)


def test_prefill_then_decode_steps_match_the_forward():
    from mla import FusedMLA
    from mla_cache import LatentKVCache
    import ds_kernels
    B, P, hidden, steps = 3, 200, 256, 3
    mod = _module(hidden, seed=1, max_pos=256)
    fused = FusedMLA(mod, device=torch.device("cuda"))
    g = torch.Generator().manual_seed(2)
    x = torch.randn(B, P + steps, hidden, generator=g).to(torch.bfloat16)
    cache = LatentKVCache(B, 256)
    out = fused.prefill(x[:, :P].cuda(), cache)
    assert cache.current_len == P
    check(out[:, -1], _rows(mod, x[:, :P].float(), torch.tensor([P - 1]))[:, 0])
    # the cache holds the prompt's raw latents and k_pe (x @ kv_a^T, before norm and RoPE)
    lat, kpe = cache.get()
    ref_ckv = x[:, :P].float() @ mod.kv_a_proj_with_mqa.weight.t()
    check(lat, ref_ckv[..., :512], atol=3e-2)
    check(kpe, ref_ckv[..., 512:], atol=3e-2)
    for i in range(steps):
        L = P + i
        y = fused.decode(x[:, L].cuda(), cache)
        assert y.shape == (B, hidden) and cache.current_len == L + 1
        check(y, _rows(mod, x[:, :L + 1].float(), torch.tensor([L]))[:, 0])
    assert ds_kernels.device_status() == ds_kernels.DS_OK


@pytest.mark.parametrize("L", [0, 1, 63, 64, 65, 127, 128, 129, 300])
def test_decode_at_chunk_boundaries_from_update(L):
    # positions written through update() (the reference API: raw values only) get their
    # side arrays on the next decode step
    from mla import FusedMLA
    from mla_cache import LatentKVCache
    B, hidden = 2, 128
    mod = _module(hidden, seed=3 + L, max_pos=512, scaling=1.0)
    fused = FusedMLA(mod, device=torch.device("cuda"))
    g = torch.Generator().manual_seed(L)
    x = torch.randn(B, L + 1, hidden, generator=g).to(torch.bfloat16)
    cache = LatentKVCache(B, 512)
    if L:
        ckv = (x[:, :L].float() @ mod.kv_a_proj_with_mqa.weight.t()).to(torch.bfloat16)
        cache.update(ckv[..., :512].cuda(), ckv[..., 512:].cuda())
    y = fused.decode(x[:, L].cuda(), cache)
    lat, kpe = cache.get(L)
    ref = oracle.mla_decode_step(x[:, L], lat.cpu(), kpe.cpu(), mod.q_proj.weight,
                                 mod.kv_a_proj_with_mqa.weight, mod.kv_a_layernorm.weight,
                                 mod.kv_b_proj.weight, mod.o_proj.weight,
                                 mod.rotary_emb.cos_cached, mod.rotary_emb.sin_cached,
                                 mod.softmax_scale, HEADS)
    check(y, ref)


def test_decode_config4_shape():
    from mla import FusedMLA
    from mla_cache import LatentKVCache
    import ds_kernels
    B, L, hidden = 64, 2048, 2048
    mod = _module(hidden, seed=4, max_pos=L + 64, scaling=1.0, std=0.02)
    fused = FusedMLA(mod, device=torch.device("cuda"))
    g = torch.Generator(device="cuda").manual_seed(5)
    cache = LatentKVCache.for_inference(B, max_seq=L + 64)
    cache.update(torch.randn(B, L, 512, generator=g, device="cuda").to(torch.bfloat16),
                 torch.randn(B, L, 64, generator=g, device="cuda").to(torch.bfloat16))
    x = torch.randn(B, hidden, generator=g, device="cuda").to(torch.bfloat16)
    y = fused.decode(x, cache)
    torch.cuda.synchronize()
    assert ds_kernels.device_status() == ds_kernels.DS_OK
    for b in (0, 17, 63):
        lat, kpe = cache.get(L)
        ref = oracle.mla_decode_step(x[b:b + 1].cpu(), lat[b:b + 1].cpu(), kpe[b:b + 1].cpu(),
                                     mod.q_proj.weight, mod.kv_a_proj_with_mqa.weight,
                                     mod.kv_a_layernorm.weight, mod.kv_b_proj.weight,
                                     mod.o_proj.weight, mod.rotary_emb.cos_cached,
                                     mod.rotary_emb.sin_cached, mod.softmax_scale, HEADS)
        check(y[b:b + 1], ref)
