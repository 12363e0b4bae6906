"""End-to-end parity of the fused MoE layer (FusedMoELayer / fused_moe_forward /
ds_kernels.moe_layer_forward) against the f32 CPU oracle of DeepSeekMoE.forward.  Mirrors
tests/test_fused_moe_e2e.py of the reference (T in {1, 4, 16, 32, 128}, x = randn*0.1, both
APIs) and adds shared experts and the BASELINE config 0 / config 2 shapes.

The oracle routes from the router logits the device produced (copied back), so the integer
routing is defined on the same f32 values; the device routing indices must then match the
oracle bit for bit.  bf16 output tolerance: max-abs <= 2e-2 and rel-L2 <= 1e-2 (BASELINE).
"""
import pytest
import torch
import torch.nn.functional as F

import oracle
from oracle.modules import OracleMoE

pytestmark = pytest.mark.gpu

H, I, E, K = 2048, 1408, 64, 6


def rel_l2(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return (torch.linalg.vector_norm(a - b) / torch.linalg.vector_norm(b).clamp_min(1e-30)).item()


_WEIGHTS = {}


def weights(seed, n_shared):
    key = (seed, n_shared)
    if key not in _WEIGHTS:
        _WEIGHTS.clear()
        _WEIGHTS[key] = oracle.make_moe_weights(seed, H, I, E, n_shared)
    return _WEIGHTS[key]


def device_weights(W):
    dev = {
        "gate": W.gate.cuda(),
        "w1": W.w1.to(torch.bfloat16).cuda(),
        "w2": W.w2.to(torch.bfloat16).cuda(),
        "sw1": None if W.shared_w1 is None else W.shared_w1.to(torch.bfloat16).cuda(),
        "sw2": None if W.shared_w2 is None else W.shared_w2.to(torch.bfloat16).cuda(),
    }
    return dev


def run_layer(W, D, x):
    import ds_kernels
    xd = x.cuda()
    logits = F.linear(xd.float(), D["gate"])
    out = ds_kernels.moe_layer_forward(logits, xd, D["w1"], D["w2"], D["sw1"], D["sw2"], top_k=K)
    ref = oracle.moe_forward(x, W, K, logits=logits.cpu())
    return out, ref, logits


def check(out, ref, atol=2e-2):
    d = (out.float().cpu() - ref).abs().max().item()
    r = rel_l2(out, ref)
    assert d <= atol and r <= 1e-2, (d, r)


@pytest.mark.parametrize("T", [1, 4, 16, 32, 128])
def test_layer_shared_experts(T):
    W = weights(0, 2)
    D = device_weights(W)
    g = torch.Generator().manual_seed(T)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    out, ref, _ = run_layer(W, D, x)
    assert out.shape == (T, H) and out.dtype == torch.bfloat16
    check(out, ref)


def test_cfg0_full():
    # T=256, x ~ N(0,1), weights N(0, 0.02^2), seed 0, 2 shared experts
    W = weights(0, 2)
    D = device_weights(W)
    g = torch.Generator().manual_seed(0)
    x = torch.randn(256, H, generator=g).to(torch.bfloat16)
    out, ref, logits = run_layer(W, D, x)
    check(out, ref)
    import ds_kernels
    idx, w, counts = ds_kernels.moe_routing(logits, top_k=K)
    ridx, rw = oracle.route(logits.cpu(), K)
    assert torch.equal(idx.cpu(), ridx)


def test_fused_layer_module_api_and_functional_api():
    # reference e2e test shape: no shared experts, x = randn * 0.1
    import ds_kernels
    W = weights(7, 0)
    mod = OracleMoE(W, top_k=K).to(torch.bfloat16).cuda()
    from moe_fused import FusedMoELayer, fused_moe_forward
    fused = FusedMoELayer(mod)
    for T in (1, 4, 16, 32, 128):
        g = torch.Generator().manual_seed(42 + T)
        x = (torch.randn(T, H, generator=g) * 0.1).to(torch.bfloat16)
        logits = torch.empty(T, E, device="cuda")
        out = fused(x.cuda(), logits_out=logits)
        ref = oracle.moe_forward(x, W, K, logits=logits.cpu())
        assert out.shape == (T, H)
        check(out, ref, atol=2e-2)
        # the device logits are the f32 router logits up to summation order
        torch.testing.assert_close(logits.cpu(), x.float() @ W.gate.t(), atol=1e-4, rtol=1e-4)
        out2 = fused_moe_forward(x.cuda(), mod.gate.weight, list(mod.experts), top_k=K)
        assert torch.equal(out2, out)  # same router, same pipeline (no shared expert here)


def run_layer_from_x(W, D, x):
    import ds_kernels
    xd = x.cuda()
    split = ds_kernels.router_weight_split(D["gate"])
    logits = torch.empty(x.shape[0], E, device="cuda")
    out = ds_kernels.moe_layer_forward_from_x(xd, split, E, D["w1"], D["w2"], D["sw1"], D["sw2"],
                                              top_k=K, logits_out=logits)
    ref = oracle.moe_forward(x, W, K, logits=logits.cpu())
    return out, ref, logits


@pytest.mark.parametrize("T", [1, 3, 129, 1000])
def test_layer_from_x(T):
    W = weights(0, 2)
    D = device_weights(W)
    g = torch.Generator().manual_seed(500 + T)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    out, ref, logits = run_layer_from_x(W, D, x)
    check(out, ref)
    torch.testing.assert_close(logits.cpu(), x.float() @ W.gate.t(), atol=1e-4, rtol=1e-4)


def test_moe_layer_fused_equals_from_x():
    import ds_kernels
    W = weights(0, 2)
    D = device_weights(W)
    g = torch.Generator().manual_seed(901)
    x = torch.randn(333, H, generator=g).to(torch.bfloat16).cuda()
    a = ds_kernels.moe_layer_fused(x, D["gate"], D["w1"], D["w2"], D["sw1"], D["sw2"], top_k=K)
    split = ds_kernels.router_weight_split(D["gate"])
    b = ds_kernels.moe_layer_forward_from_x(x, split, E, D["w1"], D["w2"], D["sw1"], D["sw2"],
                                            top_k=K)
    assert torch.equal(a, b)


def test_cfg2_full_size_from_x():
    # The layer's own routing (router GEMM partials -> route kernel, inside the one C call) is
    # read back from its workspace and must equal the oracle's routing of the device logits
    # index for index at the full config-2 size; weights at 1e-6; then the output bound.
    import ds_kernels
    from moe_fused import FusedMoELayer
    W = weights(1, 2)
    D = device_weights(W)
    g = torch.Generator().manual_seed(1002)
    x = torch.randn(8192, H, generator=g).to(torch.bfloat16)
    layer = FusedMoELayer.from_packed(D["gate"], D["w1"], D["w2"], D["sw1"], D["sw2"], top_k=K)
    logits = torch.empty(8192, E, device="cuda")
    out = layer(x.cuda(), logits_out=logits)
    idx, w = layer.last_routing(8192)
    ridx, rw = oracle.route(logits.cpu(), K)
    assert torch.equal(idx.cpu(), ridx)
    torch.testing.assert_close(w.cpu(), rw, atol=1e-6, rtol=0)
    ref = oracle.moe_forward(x, W, K, logits=logits.cpu())
    check(out, ref)
    out2, _, _ = run_layer_from_x(W, D, x)
    assert torch.equal(out, out2)


def test_layer_deterministic():
    W = weights(0, 2)
    D = device_weights(W)
    g = torch.Generator().manual_seed(3)
    x = torch.randn(512, H, generator=g).to(torch.bfloat16)
    a, _, _ = run_layer(W, D, x)
    b, _, _ = run_layer(W, D, x)
    assert torch.equal(a, b)


def test_cfg2_full_size():
    # T=8192, seed 1, 64 experts + 2 shared, x ~ N(0, 1)
    W = weights(1, 2)
    D = device_weights(W)
    g = torch.Generator().manual_seed(1001)
    x = torch.randn(8192, H, generator=g).to(torch.bfloat16)
    out, ref, logits = run_layer(W, D, x)
    check(out, ref)


class _NoOut(torch.nn.Module):
    """A layer whose forward takes no `out=`: the pipeline keeps each result alive instead."""

    def __init__(self, layer):
        super().__init__()
        self.layer = layer

    def forward(self, x):
        return self.layer(x)


@pytest.mark.parametrize("takes_out", [True, False])
def test_host_pipeline_matches_direct_calls(takes_out):
    # moe_fused.HostPipeline: pinned host batches -> device -> layer -> pinned host, with the
    # copies overlapped across batches; results must equal direct device calls bit for bit,
    # whether the layer writes into the pipeline's per-slot outputs or returns its own.
    from moe_fused import FusedMoELayer, HostPipeline
    W = weights(0, 2)
    D = device_weights(W)
    layer = FusedMoELayer.from_packed(D["gate"], D["w1"], D["w2"], D["sw1"], D["sw2"], top_k=K)
    g = torch.Generator().manual_seed(77)
    xs = [torch.randn(T, H, generator=g).to(torch.bfloat16).pin_memory()
          for T in (300, 512, 1, 300, 7, 512)]
    outs = [torch.empty(x.shape, dtype=torch.bfloat16).pin_memory() for x in xs]
    pipe = HostPipeline(layer if takes_out else _NoOut(layer), max_tokens=512, hidden=H)
    assert pipe.takes_out == takes_out
    for x, o in zip(xs, outs):
        pipe.submit(x, o)
    pipe.synchronize()
    for x, o in zip(xs, outs):
        assert torch.equal(o, layer(x.cuda()).cpu())
