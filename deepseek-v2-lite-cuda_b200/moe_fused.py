"""Fused MoE forward (drop-in for src/kernels/moe_fused.py).

Public API kept from the reference:
  FusedMoELayer(moe_module)                      (moe_fused.py:161-216)
  fused_moe_forward(hidden_states, gate_weight, experts, top_k=6, packed_w1=None, w2=None)
                                                 (moe_fused.py:227-272)

Per call: ONE C-ABI call (ds_moe_layer_forward_from_x) that runs the router (x @ gate^T with
f32 accuracy on the tensor cores: the f32 gate is pre-split into three bf16 parts that sum
to it exactly; the GEMM epilogue does the top-k and softmax) -> plan -> dispatch -> tcgen05
grouped GEMM1 with fused SwiGLU -> grouped GEMM2 -> (shared expert) -> combine on the
current stream, with no host synchronisation and no Python loop over experts.  The
reference computes the router as F.linear(x.float(), W.float()) (moe_fused.py:131).

Difference from the reference: FusedMoELayer also runs the module's shared experts
(src/reference/moe.py:72-74,106-107), which the reference pipeline drops, so its output
equals DeepSeekMoE.forward for any n_shared_experts.
"""
from __future__ import annotations

import inspect
from typing import Optional

import torch
import torch.nn as nn

import ds_kernels
from expert_prepack import prepack_experts, prepack_shared


class _Workspace:
    """Grow-only device workspace reused across calls on one device/stream."""

    def __init__(self):
        self.buf: Optional[torch.Tensor] = None

    def get(self, nbytes: int, device: torch.device) -> torch.Tensor:
        if self.buf is None or self.buf.numel() < nbytes or self.buf.device != device:
            self.buf = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device)
        return self.buf


def _layer(hidden_states, router_w_split, num_experts, packed_w1, w2, shared_w1, shared_w2,
           top_k, ws, events=None, logits_out=None, out=None):
    T, H = hidden_states.shape
    E, twoI, _ = packed_w1.shape
    Is = 0 if shared_w1 is None else shared_w1.shape[0] // 2
    need = ds_kernels.moe_layer_workspace_size(T, H, E, top_k, twoI // 2, Is)
    return ds_kernels.moe_layer_forward_from_x(hidden_states, router_w_split, num_experts,
                                               packed_w1, w2, shared_w1, shared_w2, top_k=top_k,
                                               workspace=ws.get(need, hidden_states.device),
                                               events=events, logits_out=logits_out, out=out)


class FusedMoELayer(nn.Module):
    """Drop-in replacement for DeepSeekMoE running the fused sm_100a pipeline.

    Reads `gate.weight`, `num_experts_per_tok`, `experts` and (if present and not None)
    `shared_experts` from `moe_module`; expert weights are pre-packed once.
    """

    def __init__(self, moe_module: nn.Module, verbose: bool = False):
        super().__init__()
        if not hasattr(moe_module, "gate") or not hasattr(moe_module, "experts"):
            raise ValueError(
                "FusedMoELayer: moe_module must have 'gate' and 'experts' attributes.")
        self.gate_weight = moe_module.gate.weight.detach()
        self.top_k = moe_module.num_experts_per_tok
        self.num_experts = len(moe_module.experts)
        self.packed_w1, self.w2 = prepack_experts(list(moe_module.experts))
        self.router_w_split = ds_kernels.router_weight_split(
            self.gate_weight.to(self.packed_w1.device))
        shared = getattr(moe_module, "shared_experts", None)
        if shared is not None:
            self.shared_w1, self.shared_w2 = prepack_shared(shared, self.packed_w1.device)
        else:
            self.shared_w1 = self.shared_w2 = None
        self._ws = _Workspace()
        if verbose:
            print(f"[FusedMoELayer] packed_w1 {tuple(self.packed_w1.shape)} "
                  f"w2 {tuple(self.w2.shape)} shared={'yes' if shared is not None else 'no'}")

    @classmethod
    def from_packed(cls, gate_weight: torch.Tensor, packed_w1: torch.Tensor, w2: torch.Tensor,
                    shared_w1: Optional[torch.Tensor] = None,
                    shared_w2: Optional[torch.Tensor] = None, top_k: int = 6) -> "FusedMoELayer":
        """Build from weights already in the packed layout (expert_prepack.py contract):
        gate [E, H], packed_w1 bf16 [E, 2I, H], w2 bf16 [E, H, I], shared_w1 bf16 [2Is, H],
        shared_w2 bf16 [H, Is]."""
        self = cls.__new__(cls)
        nn.Module.__init__(self)
        self.gate_weight = gate_weight.detach()
        self.top_k = top_k
        self.num_experts = packed_w1.shape[0]
        self.packed_w1, self.w2 = packed_w1.contiguous(), w2.contiguous()
        self.shared_w1 = None if shared_w1 is None else shared_w1.contiguous()
        self.shared_w2 = None if shared_w2 is None else shared_w2.contiguous()
        self.router_w_split = ds_kernels.router_weight_split(gate_weight.to(packed_w1.device))
        self._ws = _Workspace()
        return self

    def last_routing(self, num_tokens: int):
        """(topk_indices int32 [T, k], topk_weights f32 [T, k]) of the last forward over
        `num_tokens` tokens, read from the layer's workspace (valid until the next forward)."""
        Is = 0 if self.shared_w1 is None else self.shared_w1.shape[0] // 2
        idx, w, _ = ds_kernels.moe_layer_workspace_routing(
            self._ws.buf, num_tokens, self.packed_w1.shape[2], self.num_experts, self.top_k,
            self.packed_w1.shape[1] // 2, Is)
        return idx, w

    def forward(self, hidden_states: torch.Tensor, events=None,
                logits_out: Optional[torch.Tensor] = None,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """hidden_states bf16 [T, H] -> bf16 [T, H] (into `out` when given).  `logits_out`
        (f32 [T, E]) receives the router logits; `events` (9 CUDA events) are recorded between
        the phases."""
        assert hidden_states.is_cuda, "hidden_states must be on CUDA."
        assert hidden_states.dtype == torch.bfloat16, "hidden_states must be BF16."
        assert hidden_states.dim() == 2, "hidden_states must be 2-D [T, H]."
        return _layer(hidden_states.contiguous(), self.router_w_split, self.num_experts,
                      self.packed_w1, self.w2, self.shared_w1, self.shared_w2, self.top_k,
                      self._ws, events, logits_out, out)


_WEIGHT_CACHE: dict = {}
_FN_WS = _Workspace()


def fused_moe_forward(hidden_states: torch.Tensor, gate_weight: torch.Tensor, experts: list,
                      top_k: int = 6, packed_w1: Optional[torch.Tensor] = None,
                      w2: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Functional fused MoE forward (routed experts only, as the reference function).

    Pre-packs `experts` on first use and caches the result keyed by id(experts).
    """
    assert hidden_states.is_cuda, "hidden_states must be on CUDA."
    assert hidden_states.dim() == 2, "hidden_states must be [num_tokens, hidden_size]."
    assert hidden_states.dtype == torch.bfloat16, "hidden_states must be BF16."
    if packed_w1 is None or w2 is None:
        key = id(experts)
        if key not in _WEIGHT_CACHE:
            _WEIGHT_CACHE[key] = prepack_experts(experts)
        packed_w1, w2 = _WEIGHT_CACHE[key]
    split = ds_kernels.router_weight_split(gate_weight.to(hidden_states.device))
    return _layer(hidden_states.contiguous(), split, gate_weight.shape[0], packed_w1, w2, None,
                  None, top_k, _FN_WS)


class HostPipeline:
    """Streams batches that live in pinned host memory through a layer and back.

    Each submitted batch is copied host->device on a copy stream, run through the layer on the
    compute stream, and copied device->host on a second copy stream, so the copies of one
    batch overlap the compute of its neighbours (the copy engines and the SMs work
    concurrently).  Every batch still makes its own round trip.  Input and output buffers are
    allocated once per slot (a layer whose forward takes `out=` writes into its slot), so a
    steady stream of batches allocates no device memory: an allocation in the loop could
    synchronise the device and stall the pipeline.

        pipe = HostPipeline(layer, max_tokens=8192, hidden=2048)
        for x_host, out_host in batches:          # pinned CPU bf16 tensors [T, H]
            pipe.submit(x_host, out_host)
        pipe.synchronize()                        # every out_host now holds its result
    """

    def __init__(self, layer: nn.Module, max_tokens: int, hidden: int,
                 device: Optional[torch.device] = None, depth: int = 2):
        dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.layer = layer
        self.depth = depth
        self.compute = torch.cuda.current_stream(dev)
        self.h2d = torch.cuda.Stream(dev)
        self.d2h = torch.cuda.Stream(dev)
        self.x = [torch.empty((max_tokens, hidden), dtype=torch.bfloat16, device=dev)
                  for _ in range(depth)]
        self.takes_out = "out" in inspect.signature(layer.forward).parameters
        self.out = [torch.empty((max_tokens, hidden), dtype=torch.bfloat16, device=dev)
                    for _ in range(depth)] if self.takes_out else None
        self.out_free = [torch.cuda.Event() for _ in range(depth)]
        self.in_ready = [torch.cuda.Event() for _ in range(depth)]
        self.x_free = [torch.cuda.Event() for _ in range(depth)]
        self.out_ready = [torch.cuda.Event() for _ in range(depth)]
        self.used = [False] * depth
        self.n = 0

    def submit(self, x_host: torch.Tensor, out_host: torch.Tensor) -> None:
        i = self.n % self.depth
        T = x_host.shape[0]
        xb = self.x[i][:T]
        if self.used[i]:  # the slot's previous batch must be consumed by the layer first
            self.h2d.wait_event(self.x_free[i])
        with torch.cuda.stream(self.h2d):
            xb.copy_(x_host, non_blocking=True)
            self.in_ready[i].record(self.h2d)
        self.compute.wait_event(self.in_ready[i])
        with torch.cuda.stream(self.compute):
            if self.takes_out:
                if self.used[i]:  # the slot's previous output has been copied out
                    self.compute.wait_event(self.out_free[i])
                out = self.layer(xb, out=self.out[i][:T])
            else:
                out = self.layer(xb)
            self.x_free[i].record(self.compute)
            self.out_ready[i].record(self.compute)
        self.d2h.wait_event(self.out_ready[i])
        with torch.cuda.stream(self.d2h):
            out_host.copy_(out, non_blocking=True)
            if self.takes_out:
                self.out_free[i].record(self.d2h)
            else:
                out.record_stream(self.d2h)
        self.used[i] = True
        self.n += 1

    def synchronize(self) -> None:
        self.d2h.synchronize()
        self.compute.synchronize()
