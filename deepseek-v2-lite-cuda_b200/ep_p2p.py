"""Expert-parallel DeepSeek-V2-Lite MoE layer over NVLink peer memory (one process per GPU).

Rank r of N owns experts [r*E/N, (r+1)*E/N) and its own tokens, as in ep_moe.EPMoELayer,
but the three exchanges run inside the layer's own kernels instead of NCCL all-to-alls:
every rank allocates one symmetric segment (count matrix, per-forward flags, receive rows,
return rows), the segments are mapped into every rank's address space with CUDA IPC once at
construction, and each forward is one C call (ds_ep_layer_forward):

  route | plan + count exchange | dispatch straight into the owners' receive buffers,
  with the shared expert's GEMM1+SwiGLU beside it on a side stream |
  routed GEMM1+SwiGLU (once all ranks' rows are in) |
  GEMM2 (routed rows stored straight back to the token owners, then the shared expert) |
  combine (after all ranks returned their rows)

with no host synchronisation and no collective call on the data path.  Every rank must call
forward the same number of times (T may differ per rank, 0 included).  Each routed expert
row is computed by the same kernel as on one GPU, so the output equals the single-GPU layer's
bit for bit.

The reference has no multi-GPU code; this is the sharding the expert-parallel configuration
asks for (contiguous expert partition, T tokens per rank).
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

import ds_kernels


class P2PEPMoELayer(torch.nn.Module):
    """gate_weight [E, H] (all experts), packed_w1_local bf16 [E/N, 2I, H], w2_local bf16
    [E/N, H, I] for this rank's experts, shared expert weights (replicated) or None.
    forward(x [T, H] bf16, T <= max_tokens) -> [T, H] bf16.  With no process group (or world
    size 1) the layer runs the same protocol on one GPU."""

    PHASES = ("route", "plan_exchange", "dispatch_send", "gemm1", "gemm2_return", "combine")

    def __init__(self, gate_weight: torch.Tensor, packed_w1_local: torch.Tensor,
                 w2_local: torch.Tensor, shared_w1: Optional[torch.Tensor] = None,
                 shared_w2: Optional[torch.Tensor] = None, top_k: int = 6,
                 max_tokens: int = 8192, group: Optional[dist.ProcessGroup] = None,
                 timeout_ms: int = 10000):
        super().__init__()
        if dist.is_available() and dist.is_initialized():
            self.world = dist.get_world_size(group)
            self.rank = dist.get_rank(group)
        else:
            self.world, self.rank = 1, 0
        self.group = group
        self.device = packed_w1_local.device
        if self.device.type != "cuda":
            raise RuntimeError("P2PEPMoELayer needs CUDA tensors")
        self.num_experts, self.hidden = gate_weight.shape
        if self.num_experts % self.world != 0:
            raise ValueError(f"num_experts {self.num_experts} not divisible by world {self.world}")
        self.local_experts = self.num_experts // self.world
        if packed_w1_local.shape[0] != self.local_experts:
            raise ValueError("packed_w1_local must hold num_experts / world experts")
        self.w1 = packed_w1_local.contiguous()
        self.w2 = w2_local.contiguous()
        self.shared_w1 = shared_w1
        self.shared_w2 = shared_w2
        self.top_k = top_k
        self.max_tokens = max_tokens
        self.timeout_ms = timeout_ms
        self.router_w_split = ds_kernels.router_weight_split(gate_weight.to(self.device))
        I = self.w1.shape[1] // 2
        Is = 0 if shared_w1 is None else shared_w1.shape[0] // 2
        self.workspace = torch.empty(
            max(1, ds_kernels.ep_layer_workspace_size(max_tokens, self.hidden, self.num_experts,
                                                      top_k, I, Is, self.world)),
            dtype=torch.uint8, device=self.device)
        nbytes = ds_kernels.ep_symmetric_size(max_tokens, self.hidden, self.num_experts, top_k,
                                              self.world)
        self._segment = ds_kernels.ep_alloc(nbytes, self.device)
        self._peers = {}
        bases = [0] * self.world
        bases[self.rank] = self._segment
        if self.world > 1:
            h = ds_kernels.ep_ipc_handle(self._segment, self.device)
            mine = torch.tensor(list(h), dtype=torch.uint8, device=self.device)
            every = torch.empty(self.world * len(h), dtype=torch.uint8, device=self.device)
            dist.all_gather_into_tensor(every, mine, group=group)
            every = bytes(every.cpu().tolist())
            n = len(h)
            for r in range(self.world):
                if r != self.rank:
                    self._peers[r] = ds_kernels.ep_ipc_open(every[r * n:(r + 1) * n], self.device)
                    bases[r] = self._peers[r]
            self._barrier()  # every rank mapped every segment before any forward writes
        self.sym_bases = bases
        self._epoch = 0

    def _barrier(self):
        if self.world > 1:
            if dist.get_backend(self.group) == "nccl":
                dist.barrier(group=self.group, device_ids=[self.device.index])
            else:
                dist.barrier(group=self.group)

    def forward(self, x: torch.Tensor, events=None,
                logits_out: Optional[torch.Tensor] = None,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if self._segment is None:
            raise RuntimeError("P2PEPMoELayer: closed")
        if x.shape[0] > self.max_tokens:
            raise RuntimeError(f"P2PEPMoELayer: {x.shape[0]} tokens > max_tokens {self.max_tokens}")
        self._epoch += 1
        return ds_kernels.ep_layer_forward(
            x, self.router_w_split, self.num_experts, self.w1, self.w2, self.shared_w1,
            self.shared_w2, self.top_k, self.rank, self.world, self.max_tokens, self.sym_bases,
            self._epoch, self.workspace, out=out, timeout_ms=self.timeout_ms, events=events,
            logits_out=logits_out)

    def check(self) -> None:
        """Synchronise and raise if a bounded cross-GPU wait of an earlier forward ran out
        (the layer must then be closed and re-created on every rank)."""
        torch.cuda.synchronize(self.device)
        with torch.cuda.device(self.device):
            st = ds_kernels.device_status()
        if st != ds_kernels.DS_OK:
            raise RuntimeError(f"P2PEPMoELayer: device status {st} (a cross-GPU wait ran out)")

    def close(self) -> None:
        """Unmap the peers' segments and free this rank's (collective when world > 1)."""
        if self._segment is None:
            return
        torch.cuda.synchronize(self.device)
        self._barrier()  # no rank still writes into a segment that is about to go
        for p in self._peers.values():
            ds_kernels.ep_ipc_close(p, self.device)
        self._peers = {}
        self._barrier()  # every mapping of this rank's segment is closed
        ds_kernels.ep_free(self._segment, self.device)
        self._segment = None
