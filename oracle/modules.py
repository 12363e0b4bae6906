"""nn.Module view of the oracle with the attribute layout of the reference DeepSeekMoE
(src/reference/moe.py:45-75): `gate.weight`, `num_experts_per_tok`, `experts[i].{gate,up,
down}_proj`, `shared_experts` — so FusedMoELayer(moe_module) can be built from it in tests.
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
