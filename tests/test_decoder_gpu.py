"""DeepSeek-V2-Lite decoder stack (decoder.FusedDecoderStack) against a composed f32 oracle.

Three pre-norm layers (src/reference/decoder_layer.py:123-139): layer 0 with the dense SwiGLU
FFN, layers 1-2 with the MoE block (64-expert geometry reduced: 16 experts, top-4, one shared
expert), reduced hidden size, the real MLA head sizes.  prefill() over a prompt fills one
latent KV cache per layer; two decode_step() calls follow.  The oracle runs the whole token
sequence through each layer in f32 (oracle.mla_forward, oracle.moe_forward,
oracle.dense_mlp, RMSNorm) and the decode outputs must match its last rows; the prefill
output its rows; then the same decode step through the stack's CUDA graph (positions read
from the caches' device-side lengths) must continue the sequence.  Bound: rel-L2 <= 1e-2
and max-abs <= 2.5e-2 x max|ref| (three layers of bf16 activations of magnitude ~4, and a
routing near-tie can pick a different low-weight expert)."""
import math

import pytest
import torch

import oracle
from oracle.moe_oracle import MoEWeights

pytestmark = pytest.mark.gpu

H, HEADS, E, K, I_MOE, I_DENSE = 256, 16, 16, 4, 128, 512


def check(out, ref, rel=1e-2):
    o, r = out.float().cpu(), ref.float().cpu()
    d = (o - r).abs().max().item()
    e = ((o - r).norm() / r.norm()).item()
    assert d <= 2.5e-2 * r.abs().max().item() and e <= rel, (d, e, r.abs().max().item())


def _w(g, *shape, std=0.02):
    return (torch.randn(*shape, generator=g) * std).to(torch.bfloat16).float()


def _build(seed=0, positions=128):
    import decoder
    from decoder import DenseFFN, FusedDecoderLayer, FusedDecoderStack
    from mla import FusedMLA
    from moe_fused import FusedMoELayer
    g = torch.Generator().manual_seed(seed)
    cos, sin, scale = decoder.yarn_tables(positions, 40.0, "cpu")
    layers, ref_layers = [], []
    for i in range(3):
        mla_w = dict(w_q=_w(g, HEADS * 192, H), w_kva=_w(g, 576, H),
                     norm_w=torch.rand(512, generator=g) + 0.5, w_kvb=_w(g, HEADS * 256, 512),
                     w_o=_w(g, H, HEADS * 128))
        w_in = torch.rand(H, generator=g) + 0.5
        w_post = torch.rand(H, generator=g) + 0.5
        if i == 0:
            ffn_w = dict(w1=_w(g, 2 * I_DENSE, H, std=0.05), w2=_w(g, H, I_DENSE, std=0.05))
            ffn = DenseFFN(ffn_w["w1"].to(torch.bfloat16).cuda(), ffn_w["w2"].to(torch.bfloat16).cuda())
            ref_ffn = lambda x, fw=ffn_w: oracle.dense_mlp(x, fw["w1"], fw["w2"])  # noqa: E731
        else:
            W = MoEWeights(_w(g, E, H, std=0.5), _w(g, E, 2 * I_MOE, H, std=0.05),
                           _w(g, E, H, I_MOE, std=0.05), _w(g, 2 * I_MOE, H, std=0.05),
                           _w(g, H, I_MOE, std=0.05))
            ffn = FusedMoELayer.from_packed(W.gate.cuda(), W.w1.to(torch.bfloat16).cuda(),
                                            W.w2.to(torch.bfloat16).cuda(),
                                            W.shared_w1.to(torch.bfloat16).cuda(),
                                            W.shared_w2.to(torch.bfloat16).cuda(), top_k=K)
            ref_ffn = lambda x, W=W: oracle.moe_forward(x, W, K)  # noqa: E731
        attn = FusedMLA.from_weights(*(mla_w[k].cuda() for k in ("w_q", "w_kva", "norm_w", "w_kvb", "w_o")),
                                     cos.cuda(), sin.cuda(), scale, HEADS)
        layers.append(FusedDecoderLayer(attn, ffn, w_in.cuda(), w_post.cuda()))
        ref_layers.append((mla_w, ref_ffn, w_in, w_post))
    return FusedDecoderStack(layers), ref_layers, cos.float(), sin.float(), scale


def _oracle_stack(ref_layers, x, cos, sin, scale):
    h = x.float()
    B, S, _ = h.shape
    for mla_w, ref_ffn, w_in, w_post in ref_layers:
        a = oracle.mla_forward(oracle.rms_norm(h, w_in), mla_w["w_q"], mla_w["w_kva"],
                               mla_w["norm_w"], mla_w["w_kvb"], mla_w["w_o"], cos, sin, scale,
                               HEADS)
        h = h + a
        f = ref_ffn(oracle.rms_norm(h, w_post).reshape(B * S, H)).view(B, S, H)
        h = h + f
    return h


def test_stack_prefill_then_decode():
    stack, ref_layers, cos, sin, scale = _build()
    B, P, steps, graphed = 3, 64, 2, 3
    g = torch.Generator().manual_seed(9)
    x = torch.randn(B, P + steps + 1 + graphed, H, generator=g).to(torch.bfloat16)
    caches = stack.new_caches(B, 128)
    out = stack.prefill(x[:, :P].cuda(), caches)
    ref = _oracle_stack(ref_layers, x, cos, sin, scale)
    check(out, ref[:, :P])
    for i in range(steps):
        y = stack.decode_step(x[:, P + i].cuda(), caches)
        check(y, ref[:, P + i])
    assert all(c.current_len == P + steps for c in caches)
    # the captured graph: capture_decode runs one eager step (position P+steps), replays go on
    y = stack.capture_decode(x[:, P + steps].cuda(), caches)
    check(y, ref[:, P + steps])
    for i in range(graphed):
        pos = P + steps + 1 + i
        y = stack.replay_decode(x[:, pos].cuda())
        check(y, ref[:, pos])
    assert all(c.current_len == P + steps + 1 + graphed for c in caches)
    assert all(int(c.len_dev.item()) == c.current_len for c in caches)
