"""Seeded synthetic inputs with the shapes and distributions of the BASELINE configs.

There is no network for checkpoints or datasets: benchmarks use random-init weights of the
real DeepSeek-V2-Lite MoE architecture and N(0, 1) tokens, generated on the device from a
seed in a fixed draw order (router, per expert gate/up/down, shared gate/up/down).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch


@dataclass
class LayerWeights:
    gate: torch.Tensor                 # f32 [E, H] (bf16-representable values)
    packed_w1: torch.Tensor            # bf16 [E, 2I, H], gate rows then up rows
    w2: torch.Tensor                   # bf16 [E, H, I]
    shared_w1: Optional[torch.Tensor]  # bf16 [2Is, H] or None
    shared_w2: Optional[torch.Tensor]  # bf16 [H, Is] or None


def make_layer_weights(seed: int, device, H: int = 2048, I: int = 1408, E: int = 64,
                       n_shared: int = 2, std: float = 0.02) -> LayerWeights:
    g = torch.Generator(device=device).manual_seed(seed)

    def draw(*shape):
        return (torch.randn(*shape, generator=g, device=device) * std).to(torch.bfloat16)

    gate = draw(E, H).float()
    w1 = torch.empty(E, 2 * I, H, dtype=torch.bfloat16, device=device)
    w2 = torch.empty(E, H, I, dtype=torch.bfloat16, device=device)
    for e in range(E):
        w1[e, :I] = draw(I, H)
        w1[e, I:] = draw(I, H)
        w2[e] = draw(H, I)
    sw1 = sw2 = None
    if n_shared > 0:
        Is = I * n_shared
        sw1 = torch.cat([draw(Is, H), draw(Is, H)], 0).contiguous()
        sw2 = draw(H, Is)
    return LayerWeights(gate, w1, w2, sw1, sw2)


def make_tokens(seed: int, T: int, H: int, device) -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randn(T, H, generator=g, device=device).to(torch.bfloat16)


def zipf_logits(T: int, E: int, seed: int, device) -> torch.Tensor:
    """Config 1 router logits: N(0, 1) + 2*log(1/(rank+1)), rank = expert index."""
    g = torch.Generator(device=device).manual_seed(seed)
    bias = torch.tensor([2.0 * math.log(1.0 / (r + 1)) for r in range(E)], device=device)
    return torch.randn(T, E, generator=g, device=device) + bias
