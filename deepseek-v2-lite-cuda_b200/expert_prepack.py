"""Expert weight layout contract (drop-in for src/kernels/expert_prepack.py:47-161).

packed_w1[e] = cat(gate_proj.weight, up_proj.weight)  -> bf16 [E, 2I, H] (gate rows first)
w2[e]        = down_proj.weight                        -> bf16 [E, H, I]

Both are nn.Linear [out, in] layouts, i.e. K-major operands for the tcgen05 grouped GEMM,
which reads the gate and up halves of packed_w1 as the two 128-row halves of one N tile,
so no further repacking is needed on the device.
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch
from torch import nn


def _expert_shapes(experts: List[nn.Module]) -> Tuple[int, int]:
    if len(experts) == 0:
        raise ValueError("prepack_experts: experts list is empty.")
    e0 = experts[0]
    for attr in ("gate_proj", "up_proj", "down_proj"):
        if not hasattr(e0, attr):
            raise AttributeError(
                f"prepack_experts: expert module is missing attribute '{attr}'. "
                "Expected an ExpertMLP with gate_proj, up_proj, and down_proj.")
    inter, hidden = e0.gate_proj.weight.shape
    for i, ex in enumerate(experts):
        g, u, d = ex.gate_proj.weight.shape, ex.up_proj.weight.shape, ex.down_proj.weight.shape
        assert g == (inter, hidden), \
            f"Expert {i} gate_proj shape mismatch: expected {(inter, hidden)}, got {g}"
        assert u == (inter, hidden), \
            f"Expert {i} up_proj shape mismatch: expected {(inter, hidden)}, got {u}"
        assert d == (hidden, inter), \
            f"Expert {i} down_proj shape mismatch: expected {(hidden, inter)}, got {d}"
    return inter, hidden


def prepack_experts(experts: List[nn.Module],
                    device: Optional[torch.device] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Stack E ExpertMLP modules into (packed_w1 [E, 2I, H], w2 [E, H, I]) bf16 CUDA tensors."""
    _expert_shapes(experts)
    dev = device if device is not None else experts[0].gate_proj.weight.device
    if torch.device(dev).type != "cuda":
        raise RuntimeError(
            "prepack_experts: expert weights must be on a CUDA device. "
            f"Got device: {dev}")
    with torch.no_grad():
        packed_w1 = torch.stack([
            torch.cat([ex.gate_proj.weight, ex.up_proj.weight], dim=0).to(device=dev, dtype=torch.bfloat16)
            for ex in experts]).contiguous()
        w2 = torch.stack([ex.down_proj.weight.to(device=dev, dtype=torch.bfloat16)
                          for ex in experts]).contiguous()
    return packed_w1, w2


def prepack_shared(shared: nn.Module,
                   device: Optional[torch.device] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Shared expert (one SwiGLU MLP) -> (shared_w1 [2Is, H], shared_w2 [H, Is]) bf16."""
    dev = device if device is not None else shared.gate_proj.weight.device
    with torch.no_grad():
        w1 = torch.cat([shared.gate_proj.weight, shared.up_proj.weight], dim=0)
        return (w1.to(device=dev, dtype=torch.bfloat16).contiguous(),
                shared.down_proj.weight.to(device=dev, dtype=torch.bfloat16).contiguous())


def verify_prepack(experts: List[nn.Module]) -> bool:
    """Check packed tensors against the module weights (src/kernels/expert_prepack.py:135-161)."""
    packed_w1, w2 = prepack_experts(experts)
    for i, ex in enumerate(experts):
        g = ex.gate_proj.weight.to(torch.bfloat16)
        u = ex.up_proj.weight.to(torch.bfloat16)
        d = ex.down_proj.weight.to(torch.bfloat16)
        inter = g.shape[0]
        assert torch.equal(packed_w1[i, :inter, :], g), \
            f"Expert {i}: packed_w1 gate rows do not match gate_proj.weight"
        assert torch.equal(packed_w1[i, inter:, :], u), \
            f"Expert {i}: packed_w1 up rows do not match up_proj.weight"
        assert torch.equal(w2[i], d), f"Expert {i}: w2 does not match down_proj.weight"
    return True
