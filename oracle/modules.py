"""nn.Module views of the oracle with the attribute layouts of the reference modules, so
the fused modules can be built from them in tests:

OracleMoE: DeepSeekMoE (src/reference/moe.py:45-75): `gate.weight`, `num_experts_per_tok`,
    `experts[i].{gate,up,down}_proj`, `shared_experts` -> FusedMoELayer(moe_module).
OracleMLA: DeepSeekMLA (src/reference/mla.py:209-293): `q_proj`, `kv_a_proj_with_mqa`,
    `kv_a_layernorm.{weight,variance_epsilon}`, `kv_b_proj`, `o_proj`,
    `rotary_emb.{cos_cached,sin_cached}`, `softmax_scale`, the head sizes -> FusedMLA.
Test infrastructure only (see oracle/__init__).
"""
from __future__ import annotations

import torch
from torch import nn

from .moe_oracle import MoEWeights, moe_forward


class _Gate(nn.Module):
    def __init__(self, weight: torch.Tensor):
        super().__init__()
        self.weight = nn.Parameter(weight.clone(), requires_grad=False)


class _ExpertMLP(nn.Module):
    def __init__(self, w1: torch.Tensor, w2: torch.Tensor):
        super().__init__()
        inter, hidden = w1.shape[0] // 2, w1.shape[1]
        self.gate_proj = nn.Linear(hidden, inter, bias=False)
        self.up_proj = nn.Linear(hidden, inter, bias=False)
        self.down_proj = nn.Linear(inter, hidden, bias=False)
        with torch.no_grad():
            self.gate_proj.weight.copy_(w1[:inter])
            self.up_proj.weight.copy_(w1[inter:])
            self.down_proj.weight.copy_(w2)


class OracleMoE(nn.Module):
    """DeepSeekMoE-shaped container whose forward is the f32 CPU oracle."""

    def __init__(self, W: MoEWeights, top_k: int = 6):
        super().__init__()
        self.W = W
        self.num_experts_per_tok = top_k
        self.gate = _Gate(W.gate)
        self.experts = nn.ModuleList([_ExpertMLP(W.w1[e], W.w2[e]) for e in range(W.num_experts)])
        self.shared_experts = (_ExpertMLP(W.shared_w1, W.shared_w2)
                               if W.shared_w1 is not None else None)

    def forward(self, x: torch.Tensor, logits=None) -> torch.Tensor:
        return moe_forward(x.cpu(), self.W, self.num_experts_per_tok,
                           logits=None if logits is None else logits.cpu())


class _Norm(nn.Module):
    def __init__(self, weight: torch.Tensor, eps: float):
        super().__init__()
        self.weight = nn.Parameter(weight.clone(), requires_grad=False)
        self.variance_epsilon = eps


class _Rotary(nn.Module):
    def __init__(self, cos: torch.Tensor, sin: torch.Tensor):
        super().__init__()
        self.register_buffer("cos_cached", cos.clone(), persistent=False)
        self.register_buffer("sin_cached", sin.clone(), persistent=False)


def _linear(w: torch.Tensor) -> nn.Linear:
    lin = nn.Linear(w.shape[1], w.shape[0], bias=False)
    with torch.no_grad():
        lin.weight.copy_(w)
    return lin


class OracleMLA(nn.Module):
    """DeepSeekMLA-shaped container whose forward is the f32 CPU oracle (mla_forward)."""

    def __init__(self, w_q, w_kva, norm_w, w_kvb, w_o, cos, sin, softmax_scale, heads,
                 eps: float = 1e-6):
        super().__init__()
        self.hidden_size = w_q.shape[1]
        self.num_heads = heads
        self.qk_nope_head_dim, self.qk_rope_head_dim, self.v_head_dim = 128, 64, 128
        self.kv_lora_rank = 512
        self.q_proj = _linear(w_q)
        self.kv_a_proj_with_mqa = _linear(w_kva)
        self.kv_a_layernorm = _Norm(norm_w, eps)
        self.kv_b_proj = _linear(w_kvb)
        self.o_proj = _linear(w_o)
        self.rotary_emb = _Rotary(cos, sin)
        self.softmax_scale = softmax_scale

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        from .mla_oracle import mla_forward
        return mla_forward(x.cpu(), self.q_proj.weight, self.kv_a_proj_with_mqa.weight,
                           self.kv_a_layernorm.weight, self.kv_b_proj.weight, self.o_proj.weight,
                           self.rotary_emb.cos_cached, self.rotary_emb.sin_cached,
                           self.softmax_scale, self.num_heads, self.kv_a_layernorm.variance_epsilon)
