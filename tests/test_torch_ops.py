"""The drop-in ops as torch custom operators (torch.ops.ds_kernels.*).

CPU: every op of the reference's surface (src/kernels/bindings.cu:77-192) is registered with
a schema whose argument names match the reference binding, and its fake kernel propagates
shapes and dtypes on fake CUDA tensors (no GPU needed).
GPU: torch.library.opcheck on each operator (schema, fake-vs-real agreement, AOT dispatch),
the operator returns exactly the eager function's bits, and a function calling the module's
ops compiles with torch.compile(fullgraph=True) into one graph that gives the eager result.
"""
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import ds_kernels

H, E, K, I = 256, 16, 4, 128

SURFACE = {  # op -> argument names of the reference binding
    "moe_routing": ["logits", "top_k"],
    "moe_scan": ["expert_counts"],
    "moe_dispatch": ["input", "topk_indices", "topk_weights", "expert_offsets"],
    "moe_combine": ["expert_output", "token_map", "dispatched_weights", "num_tokens"],
    "swiglu": ["input"],
    "moe_gemm1": ["dispatched", "packed_w1", "expert_offsets"],
    "moe_gemm2": ["swiglu_out", "w2", "expert_offsets"],
    "rms_norm": ["input", "weight", "eps"],
    "kv_upproj": ["normed_kv", "weight"],
    "rope": ["q_pe", "k_pe", "cos", "sin"],
}


def test_every_op_is_registered_with_the_reference_argument_names():
    for name, args in SURFACE.items():
        op = getattr(torch.ops.ds_kernels, name).default
        assert [a.name for a in op._schema.arguments] == args, name
    for extra in ("moe_gemm1_swiglu", "rms_norm_residual", "moe_layer_fused"):
        assert hasattr(torch.ops.ds_kernels, extra)


def _fake_args(dev="cuda", T=40):
    bf = torch.bfloat16
    S = T * K
    return {
        "moe_routing": ((torch.empty(T, E, device=dev), K),
                        [((T, K), torch.int32), ((T, K), torch.float32), ((E,), torch.int32)]),
        "moe_scan": ((torch.empty(E, dtype=torch.int32, device=dev),),
                     [((E + 1,), torch.int32)]),
        "moe_dispatch": ((torch.empty(T, H, dtype=bf, device=dev),
                          torch.empty(T, K, dtype=torch.int32, device=dev),
                          torch.empty(T, K, device=dev),
                          torch.empty(E + 1, dtype=torch.int32, device=dev)),
                         [((S, H), bf), ((S,), torch.int32), ((S,), torch.float32)]),
        "moe_combine": ((torch.empty(S, H, dtype=bf, device=dev),
                         torch.empty(S, dtype=torch.int32, device=dev),
                         torch.empty(S, device=dev), T), [((T, H), bf)]),
        "swiglu": ((torch.empty(S, 2 * I, dtype=bf, device=dev),), [((S, I), bf)]),
        "moe_gemm1": ((torch.empty(S, H, dtype=bf, device=dev),
                       torch.empty(E, 2 * I, H, dtype=bf, device=dev),
                       torch.empty(E + 1, dtype=torch.int32, device=dev)), [((S, 2 * I), bf)]),
        "moe_gemm1_swiglu": ((torch.empty(S, H, dtype=bf, device=dev),
                              torch.empty(E, 2 * I, H, dtype=bf, device=dev),
                              torch.empty(E + 1, dtype=torch.int32, device=dev)),
                             [((S, I), bf)]),
        "moe_gemm2": ((torch.empty(S, I, dtype=bf, device=dev),
                       torch.empty(E, H, I, dtype=bf, device=dev),
                       torch.empty(E + 1, dtype=torch.int32, device=dev)), [((S, H), bf)]),
        "rms_norm": ((torch.empty(2, T, 512, dtype=bf, device=dev),
                      torch.empty(512, device=dev), 1e-6), [((2, T, 512), bf)]),
        "rms_norm_residual": ((torch.empty(T, H, dtype=bf, device=dev),
                               torch.empty(T, H, dtype=bf, device=dev),
                               torch.empty(H, device=dev), 1e-6),
                              [((T, H), bf), ((T, H), bf)]),
        "kv_upproj": ((torch.empty(2, T, 512, dtype=bf, device=dev),
                       torch.empty(4096, 512, dtype=bf, device=dev)), [((2, T, 4096), bf)]),
        "rope": ((torch.empty(2, 16, T, 64, dtype=bf, device=dev),
                  torch.empty(2, 1, T, 64, dtype=bf, device=dev),
                  torch.empty(2, 1, T, 64, dtype=bf, device=dev),
                  torch.empty(2, 1, T, 64, dtype=bf, device=dev)),
                 [((2, 16, T, 64), bf), ((2, 1, T, 64), bf)]),
        "moe_layer_fused": ((torch.empty(T, H, dtype=bf, device=dev),
                             torch.empty(E, H, device=dev),
                             torch.empty(E, 2 * I, H, dtype=bf, device=dev),
                             torch.empty(E, H, I, dtype=bf, device=dev), None, None, K),
                            [((T, H), bf)]),
    }


def test_fake_kernels_propagate_shapes_on_fake_cuda_tensors():
    with FakeTensorMode():
        cases = _fake_args()
        for name, (args, want) in cases.items():
            out = getattr(torch.ops.ds_kernels, name)(*args)
            outs = list(out) if isinstance(out, (tuple, list)) else [out]
            got = [(tuple(t.shape), t.dtype) for t in outs]
            assert got == [(tuple(s), d) for s, d in want], name
            assert all(t.device.type == "cuda" for t in outs), name


# ------------------------------------------------------------------------------- GPU
def _real_inputs(T=300, seed=0):
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(T, E, generator=g).cuda()
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).cuda()
    w1 = (torch.randn(E, 2 * I, H, generator=g) * 0.05).to(torch.bfloat16).cuda()
    w2 = (torch.randn(E, H, I, generator=g) * 0.05).to(torch.bfloat16).cuda()
    return logits, x, w1, w2


@pytest.mark.gpu
def test_opcheck_and_bits_equal_the_eager_functions():
    logits, x, w1, w2 = _real_inputs()
    T = x.shape[0]
    idx, w, counts = ds_kernels.moe_routing(logits, top_k=K)
    off = ds_kernels.moe_scan(counts)
    disp, tm, dw = ds_kernels.moe_dispatch(x, idx, w, off)
    g1 = ds_kernels.moe_gemm1(disp, w1, off)
    h = ds_kernels.swiglu(g1)
    eo = ds_kernels.moe_gemm2(h, w2, off)
    lat = torch.randn(2, 64, 512, device="cuda").to(torch.bfloat16)
    nw = torch.rand(512, device="cuda") + 0.5
    wkv = (torch.randn(4096, 512, device="cuda") * 0.02).to(torch.bfloat16)
    q = torch.randn(2, 16, 64, 64, device="cuda").to(torch.bfloat16)
    k = torch.randn(2, 1, 64, 64, device="cuda").to(torch.bfloat16)
    cs = torch.randn(2, 1, 64, 64, device="cuda").to(torch.bfloat16)
    cases = {
        "moe_routing": (logits, K),
        "moe_scan": (counts,),
        "moe_dispatch": (x, idx, w, off),
        "moe_combine": (eo, tm, dw, T),
        "swiglu": (g1,),
        "moe_gemm1": (disp, w1, off),
        "moe_gemm1_swiglu": (disp, w1, off),
        "moe_gemm2": (h, w2, off),
        "rms_norm": (lat, nw, 1e-6),
        "rms_norm_residual": (x, x, torch.rand(H, device="cuda") + 0.5, 1e-6),
        "kv_upproj": (lat, wkv),
        "rope": (q, k, cs, cs),
    }
    for name, args in cases.items():
        op = getattr(torch.ops.ds_kernels, name)
        torch.library.opcheck(op, args)
        got = op(*args)
        want = ds_kernels._eager[name](*args)
        got = list(got) if isinstance(got, tuple) else [got]
        want = list(want) if isinstance(want, list) else [want]
        assert len(got) == len(want), name
        for a, b in zip(got, want):
            assert torch.equal(a, b), name


@pytest.mark.gpu
def test_module_ops_compile_into_one_graph():
    logits, x, w1, w2 = _real_inputs(T=257, seed=1)

    def moe_pipeline(logits, x, w1, w2):
        idx, w, counts = ds_kernels.moe_routing(logits, top_k=K)
        off = ds_kernels.moe_scan(counts)
        disp, tm, dw = ds_kernels.moe_dispatch(x, idx, w, off)
        h = ds_kernels.swiglu(ds_kernels.moe_gemm1(disp, w1, off))
        eo = ds_kernels.moe_gemm2(h, w2, off)
        return ds_kernels.moe_combine(eo, tm, dw, x.shape[0])

    torch._dynamo.reset()
    compiled = torch.compile(moe_pipeline, backend="eager", fullgraph=True)
    out = compiled(logits, x, w1, w2)
    ref = moe_pipeline(logits, x, w1, w2)
    assert torch.equal(out, ref)
