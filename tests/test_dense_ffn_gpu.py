"""DeepSeek-V2-Lite's layer-0 dense SwiGLU FFN, 2048 -> 10944 -> 2048, on the tcgen05 engine.

Layer 0 (first_k_dense_replace = 1) replaces the MoE block with one SwiGLU MLP of
intermediate size 10944 (src/reference/decoder_layer.py:8-9 notes it; the geometry is
ExpertMLP, src/reference/moe.py:6-19).  10944 = 85.5 x 128, so GEMM1's last n-tile holds 64
valid columns of each of the gate and up halves (the rest is computed and not stored);
GEMM2 runs K = 10944 = 171 k-blocks of 64.  Checked against the f32 oracle (dense_mlp) with the BASELINE float bound:
max-abs <= 2e-2 and rel-L2 <= 1e-2; weights N(0, 0.02^2), x ~ N(0, 1) as in the configs.
"""
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

H, I_DENSE = 2048, 10944

_W = {}


def weights():
    if not _W:
        g = torch.Generator().manual_seed(27)
        _W["w1"] = (torch.randn(2 * I_DENSE, H, generator=g) * 0.02).to(torch.bfloat16)
        _W["w2"] = (torch.randn(H, I_DENSE, generator=g) * 0.02).to(torch.bfloat16)
    return _W["w1"], _W["w2"]


def check(out, ref):
    o = out.float().cpu()
    d = (o - ref).abs().max().item()
    r = ((o - ref).norm() / ref.norm()).item()
    assert d <= 2e-2 and r <= 1e-2, (d, r)


@pytest.mark.parametrize("T", [1, 64, 300, 2048])
def test_layer0_dense_ffn(T):
    import ds_kernels
    w1, w2 = weights()
    g = torch.Generator().manual_seed(T)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    out = ds_kernels.dense_mlp(x.cuda(), w1.cuda(), w2.cuda())
    assert out.shape == (T, H) and out.dtype == torch.bfloat16
    check(out, oracle.dense_mlp(x, w1, w2))


def test_layer0_dense_ffn_gemm1_halves():
    # the SwiGLU intermediate alone: silu(x @ gate^T) * (x @ up^T), 10944 columns
    import ds_kernels
    w1, _ = weights()
    g = torch.Generator().manual_seed(5)
    x = torch.randn(129, H, generator=g).to(torch.bfloat16)
    h = ds_kernels.dense_gemm1_swiglu(x.cuda(), w1.cuda())
    assert h.shape == (129, I_DENSE)
    xf = x.float()
    gt = xf @ w1[:I_DENSE].float().t()
    up = xf @ w1[I_DENSE:].float().t()
    ref = gt / (1 + torch.exp(-gt)) * up
    hf = h.float().cpu()
    assert ((hf - ref).abs() <= 2e-2 + 2 ** -8 * ref.abs()).all()


@pytest.mark.parametrize("T", [1, 64, 200])
def test_layer0_dense_ffn_split_k(T):
    # few rows: dense_mlp_ws splits the K loop of both GEMMs over the SMs (f32 partials in the
    # workspace, summed in slice order, then the SwiGLU / plain epilogue)
    import ds_kernels
    w1, w2 = weights()
    g = torch.Generator().manual_seed(100 + T)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    out = ds_kernels.dense_mlp_ws(x.cuda(), w1.cuda(), w2.cuda())
    assert out.shape == (T, H)
    check(out, oracle.dense_mlp(x, w1, w2))
    assert int(ds_kernels.library().ds_dense_mlp_workspace_size(T, H, I_DENSE)) > 0
