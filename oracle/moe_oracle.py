"""CPU restatement of the reference MoE path (test infrastructure only; see oracle/__init__).

Canonical integer contract (the reference is not bit-defined for ties or slot order):
  * routing: experts ranked by f32 logit descending, equal logits -> lower expert index;
    weight = softmax value at that expert (src/reference/moe.py:33-43; softmax is monotone,
    so ranking logits ranks scores).  No renormalisation, routed_scaling_factor 1.0.
  * counts = bincount of the indices; offsets = [0] + cumsum (src/kernels/moe/scan.cu:1-16).
  * dispatch permutation: expert-major, ascending token id inside an expert — the order in
    which src/reference/moe.py:90-103 visits tokens (`mask.any(dim=1).nonzero()`).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Tuple

import torch

F32 = torch.float32


def route(logits: torch.Tensor, top_k: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """logits f32 [T, E] -> (idx int32 [T, k], w f32 [T, k]).

    src/reference/moe.py:33-43 (softmax then top-k), with the canonical tie-break above.
    """
    logits = logits.to(F32)
    order = torch.sort(-logits, dim=-1, stable=True).indices[:, :top_k]
    scores = torch.softmax(logits, dim=-1)
    w = torch.gather(scores, 1, order)
    return order.to(torch.int32), w.contiguous()


def expert_counts(idx: torch.Tensor, num_experts: int) -> torch.Tensor:
    """Per-expert token counts (src/kernels/moe/routing.cu:196-224)."""
    return torch.bincount(idx.reshape(-1).long(), minlength=num_experts).to(torch.int32)


def expert_offsets(counts: torch.Tensor) -> torch.Tensor:
    """Exclusive prefix sum with the total appended (src/kernels/moe/scan.cu:86-130)."""
    out = torch.zeros(counts.numel() + 1, dtype=torch.int64)
    out[1:] = torch.cumsum(counts.to(torch.int64), 0)
    return out.to(torch.int32)


def dispatch(x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor, num_experts: int):
    """Expert-contiguous permutation (src/kernels/moe/dispatch.cu:156-218 semantics, with the
    ascending-token order of src/reference/moe.py:95 inside each expert).

    Returns (dispatched [S, H], token_map int32 [S], dispatched_weights f32 [S],
    slot_of int32 [T, k], offsets int32 [E+1]).
    """
    T, k = idx.shape
    flat_e = idx.reshape(-1).long()
    flat_t = torch.arange(T).repeat_interleave(k)
    # stable sort by expert keeps ascending token order inside an expert
    perm = torch.sort(flat_e, stable=True).indices
    token_map = flat_t[perm].to(torch.int32)
    dweights = w.reshape(-1)[perm].to(F32)
    slot_of = torch.empty(T * k, dtype=torch.int64)
    slot_of[perm] = torch.arange(T * k)
    offsets = expert_offsets(expert_counts(idx, num_experts))
    dispatched = x[token_map.long()]
    return dispatched, token_map, dweights, slot_of.view(T, k).to(torch.int32), offsets


def combine(expert_output: torch.Tensor, token_map: torch.Tensor, dweights: torch.Tensor,
            num_tokens: int) -> torch.Tensor:
    """out[t] = sum over slots s with token_map[s] == t (ascending s) of f32(eo[s]) * w[s].

    src/kernels/moe/combine.cu:38-61 and the loop reference of
    tests/test_moe_combine_kernel.py:47-64; returns f32 [T, H] (callers round to bf16).
    """
    H = expert_output.shape[1]
    out = torch.zeros(num_tokens, H, dtype=F32)
    tm = token_map.long()
    keep = (tm >= 0) & (tm < num_tokens)
    contrib = expert_output.to(F32)[keep] * dweights.to(F32)[keep, None]
    out.index_add_(0, tm[keep], contrib)
    return out


def swiglu(x: torch.Tensor) -> torch.Tensor:
    """silu(gate) * up in f32 over [S, 2I] (src/kernels/moe/swiglu.cu:68-108)."""
    I = x.shape[1] // 2
    g = x[:, :I].to(F32)
    u = x[:, I:].to(F32)
    return g / (1.0 + torch.exp(-g)) * u


def grouped_linear(a: torch.Tensor, w: torch.Tensor, offsets: torch.Tensor) -> torch.Tensor:
    """out[off[e]:off[e+1]] = a[off[e]:off[e+1]] @ w[e]^T in f32; rows outside stay 0.

    src/kernels/moe/gemm1.cu:84-155 and gemm2.cu:75-124 (per-expert GEMM loop).
    """
    S = a.shape[0]
    N = w.shape[1]
    out = torch.zeros(S, N, dtype=F32)
    off = offsets.tolist()
    af = a.to(F32)
    for e in range(w.shape[0]):
        s0, s1 = off[e], off[e + 1]
        if s1 > s0:
            out[s0:s1] = af[s0:s1] @ w[e].to(F32).t()
    return out


@dataclass
class MoEWeights:
    """Weights of one MoE block in the packed layout (all f32 on CPU).

    gate [E, H]; w1 [E, 2I, H] (gate rows then up rows); w2 [E, H, I];
    shared_w1 [2Is, H] and shared_w2 [H, Is] or None.
    """
    gate: torch.Tensor
    w1: torch.Tensor
    w2: torch.Tensor
    shared_w1: Optional[torch.Tensor] = None
    shared_w2: Optional[torch.Tensor] = None

    @property
    def num_experts(self) -> int:
        return self.w1.shape[0]


def make_moe_weights(seed: int, H: int = 2048, I: int = 1408, E: int = 64, n_shared: int = 2,
                     std: float = 0.02, round_bf16: bool = True) -> MoEWeights:
    """Seeded synthetic weights in a fixed draw order: router, then per expert gate/up/down,
    then shared gate/up/down, each N(0, std^2) (BASELINE configs 0 and 2).  With round_bf16
    every weight is rounded to bf16 and kept as f32, so the GPU and the oracle see the same
    numbers."""
    g = torch.Generator().manual_seed(seed)

    def draw(*shape):
        t = torch.randn(*shape, generator=g, dtype=F32) * std
        return t.to(torch.bfloat16).to(F32) if round_bf16 else t

    gate = draw(E, H)
    w1 = torch.empty(E, 2 * I, H, dtype=F32)
    w2 = torch.empty(E, H, I, dtype=F32)
    for e in range(E):
        w1[e, :I] = draw(I, H)
        w1[e, I:] = draw(I, H)
        w2[e] = draw(H, I)
    sw1 = sw2 = None
    if n_shared > 0:
        Is = I * n_shared
        sw1 = torch.cat([draw(Is, H), draw(Is, H)], 0)
        sw2 = draw(H, Is)
    return MoEWeights(gate, w1, w2, sw1, sw2)


def _mlp(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor) -> torch.Tensor:
    """down(silu(gate x) * up x) with w1 = [gate; up] (src/reference/moe.py:6-19)."""
    I = w1.shape[0] // 2
    h = x @ w1.t()
    g, u = h[:, :I], h[:, I:]
    return (g / (1.0 + torch.exp(-g)) * u) @ w2.t()


def dense_mlp(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor) -> torch.Tensor:
    """Dense SwiGLU FFN in f32: down(silu(gate x) * up x), w1 = [gate; up] [2I, H], w2 [H, I].

    The geometry of ExpertMLP (src/reference/moe.py:6-19); DeepSeek-V2-Lite's layer 0 uses it
    with I = 10944 in place of the MoE block (src/reference/decoder_layer.py:8-9)."""
    return _mlp(x.to(F32), w1.to(F32), w2.to(F32))


def moe_forward(x: torch.Tensor, W: MoEWeights, top_k: int,
                logits: Optional[torch.Tensor] = None, return_aux: bool = False):
    """f32 restatement of DeepSeekMoE.forward (src/reference/moe.py:77-109).

    Routed experts are visited in ascending expert order, each over its tokens in ascending
    token order, accumulating w * expert_out into a zeroed f32 output; the shared expert is
    added last.  `logits` may be supplied (e.g. the device-produced router logits) so that
    the integer routing is defined on exactly the values the device ranked.
    """
    xf = x.to(F32)
    if logits is None:
        logits = xf @ W.gate.t()
    idx, w = route(logits, top_k)
    T = xf.shape[0]
    out = torch.zeros_like(xf)
    flat_e = idx.reshape(-1).long()
    flat_t = torch.arange(T).repeat_interleave(top_k)
    flat_w = w.reshape(-1)
    perm = torch.sort(flat_e, stable=True).indices
    counts = torch.bincount(flat_e, minlength=W.num_experts).tolist()
    pos = 0
    for e, c in enumerate(counts):
        if c == 0:
            continue
        sel = perm[pos:pos + c]
        pos += c
        toks = flat_t[sel]
        y = _mlp(xf[toks], W.w1[e], W.w2[e])
        out.index_add_(0, toks, y * flat_w[sel, None])
    if W.shared_w1 is not None:
        out += _mlp(xf, W.shared_w1, W.shared_w2)
    if return_aux:
        return out, {"logits": logits, "idx": idx, "w": w}
    return out


def zipf_logits(T: int, E: int, seed: int) -> torch.Tensor:
    """BASELINE config 1 router logits: N(0, 1) + 2*log(1/(rank+1)) with rank = expert index."""
    g = torch.Generator().manual_seed(seed)
    bias = torch.tensor([2.0 * math.log(1.0 / (r + 1)) for r in range(E)], dtype=F32)
    return torch.randn(T, E, generator=g, dtype=F32) + bias
