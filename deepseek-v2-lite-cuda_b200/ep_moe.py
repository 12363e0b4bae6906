"""Expert-parallel DeepSeek-V2-Lite MoE layer over torch.distributed (NCCL on GPUs).

Rank r of N owns experts [r*E/N, (r+1)*E/N) and its own tokens.  One forward:

  1. router logits (f32) and deterministic route+dispatch of the local tokens into an
     expert-major buffer; because experts are partitioned contiguously, that buffer is
     already grouped by destination rank (one contiguous chunk per rank);
  2. all-to-all of the per-(rank, expert) row counts (N x E/N int32), one device->host copy
     of the split sizes (the only host synchronisation);
  3. all-to-all of the dispatched rows (bf16);
  4. receive-side plan: expert-major offsets of the received rows and the row map, gather
     into expert-major order, grouped GEMM1+SwiGLU / GEMM2 on the local experts with the
     GEMM2 epilogue writing each result straight back to its source-major row;
  5. all-to-all of the expert outputs back to the token owners;
  6. combine (k expert rows per token in ascending slot order + the shared expert).

The row exchanges are issued asynchronously and the shared expert's two GEMMs run on the
compute stream while they are in flight (GEMM1 under the dispatch exchange, GEMM2 under the
return exchange), with their grid capped so NCCL's kernels keep SMs.

The reference has no multi-GPU code; this is the sharding BASELINE config 2 asks for.
The compute steps go through an `ops` object: by default the CUDA kernels of
libds_kernels_sm100.so (CudaOps); tests inject a CPU implementation to exercise this
orchestration with the gloo backend.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist


class CudaOps:
    """The layer's compute steps on the sm_100a kernels (C ABI via ds_kernels)."""

    def __init__(self):
        import ds_kernels
        self.k = ds_kernels

    def prepare_router(self, gate_weight):
        return self.k.router_weight_split(gate_weight)

    def route(self, x, router_state, num_experts, top_k, logits_out=None):
        """-> (topk_indices, topk_weights): tensor-core router with f32-accurate logits
        (written to `logits_out` f32 [T, E] when given)."""
        return self.k.moe_router(x, router_state, num_experts, top_k, logits_out=logits_out)

    def dispatch(self, idx, w, x, num_experts):
        """-> (expert_offsets, slot_of, token_map, dispatched)."""
        return self.k.moe_dispatch_routed(idx, w, x, num_experts)

    def ep_plan(self, recv_counts, recv_rows):
        return self.k.ep_plan(recv_counts, recv_rows)

    def gather_rows(self, src, row_map):
        return self.k.gather_rows(src, row_map)

    def expert_mlp(self, rows, offsets, w1, w2, out, out_row_map):
        return self.k.moe_expert_mlp(rows, offsets, w1, w2, out=out, out_row_map=out_row_map)

    def dense_mlp(self, x, w1, w2, max_ctas=0):
        return self.k.dense_mlp(x, w1, w2, max_ctas=max_ctas)

    def shared_gemm1(self, x, w1, max_ctas=0):
        """silu(x @ gate^T) * (x @ up^T) for the shared expert (GEMM1 + SwiGLU epilogue)."""
        return self.k.dense_gemm1_swiglu(x, w1, max_ctas)

    def shared_gemm2(self, h, w2, max_ctas=0):
        return self.k.dense_gemm2(h, w2, max_ctas)

    def num_sms(self, device):
        return torch.cuda.get_device_properties(device).multi_processor_count

    def combine_slots(self, back, slot_of, w, shared_out):
        return self.k.moe_combine_slots(back, slot_of, w, shared_out)


class EPMoELayer(torch.nn.Module):
    """Expert-parallel MoE layer; construct on every rank with that rank's expert slice.

    gate_weight [E, H] (all experts), packed_w1_local bf16 [E/N, 2I, H], w2_local bf16
    [E/N, H, I] for experts [rank*E/N, (rank+1)*E/N), shared expert weights (replicated)
    or None.  forward(x_local [T_r, H] bf16) -> [T_r, H] bf16.
    """

    def __init__(self, gate_weight: torch.Tensor, packed_w1_local: torch.Tensor,
                 w2_local: torch.Tensor, shared_w1: Optional[torch.Tensor] = None,
                 shared_w2: Optional[torch.Tensor] = None, top_k: int = 6,
                 group: Optional[dist.ProcessGroup] = None, ops=None):
        super().__init__()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.num_experts = gate_weight.shape[0]
        if self.num_experts % self.world != 0:
            raise ValueError(f"num_experts {self.num_experts} not divisible by world {self.world}")
        self.local_experts = self.num_experts // self.world
        if packed_w1_local.shape[0] != self.local_experts:
            raise ValueError("packed_w1_local must hold num_experts / world experts")
        self.gate_weight = gate_weight
        self.w1 = packed_w1_local.contiguous()
        self.w2 = w2_local.contiguous()
        self.shared_w1 = shared_w1
        self.shared_w2 = shared_w2
        self.top_k = top_k
        self.ops = ops if ops is not None else CudaOps()
        self.router_state = self.ops.prepare_router(gate_weight)
        self.nccl_reserve_sms = 32

    def _a2a(self, out, inp, out_splits=None, in_splits=None, async_op=False):
        return dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group,
                                      async_op=async_op)

    PHASES = ("route_dispatch", "exchange_counts", "exchange_rows", "expert_mlp",
              "exchange_back", "combine")

    def forward(self, x: torch.Tensor, events=None,
                logits_out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """events: optional list of len(PHASES)+1 CUDA events recorded on the current stream
        at the phase boundaries (for timing); logits_out (f32 [T, E]) receives the router
        logits."""
        ops, N, El, k = self.ops, self.world, self.local_experts, self.top_k

        def mark(i):
            if events is not None:
                events[i].record()
        T, H = x.shape
        has_shared = self.shared_w1 is not None
        # SMs left to NCCL while a capped GEMM overlaps an exchange
        cap = max(1, ops.num_sms(x.device) - self.nccl_reserve_sms) if x.is_cuda else 0

        mark(0)
        if logits_out is None:
            idx, w = ops.route(x, self.router_state, self.num_experts, k)
        else:
            idx, w = ops.route(x, self.router_state, self.num_experts, k, logits_out=logits_out)
        offsets, slot_of, token_map, disp = ops.dispatch(idx, w, x, self.num_experts)
        mark(1)
        counts = (offsets[1:] - offsets[:-1]).to(torch.int32).view(N, El).contiguous()
        recv_counts = torch.empty_like(counts)
        self._a2a(recv_counts, counts)
        splits = torch.cat([counts.sum(1), recv_counts.sum(1)]).cpu().tolist()
        send_splits, recv_splits = splits[:N], splits[N:]
        R = int(sum(recv_splits))
        mark(2)
        recv = torch.empty((R, H), dtype=disp.dtype, device=disp.device)
        work = self._a2a(recv, disp, recv_splits, send_splits, async_op=True)
        sh = ops.shared_gemm1(x, self.shared_w1, cap) if has_shared else None
        work.wait()
        mark(3)

        exp_off, row_map = ops.ep_plan(recv_counts, R)
        ret = torch.empty_like(recv)
        if R > 0:
            rows = ops.gather_rows(recv, row_map)
            ops.expert_mlp(rows, exp_off, self.w1, self.w2, ret, row_map)
        self.last_recv_rows = R
        mark(4)
        back = torch.empty_like(disp)
        work = self._a2a(back, ret, send_splits, recv_splits, async_op=True)
        shared_out = ops.shared_gemm2(sh, self.shared_w2, cap) if has_shared else None
        work.wait()
        mark(5)
        out = ops.combine_slots(back, slot_of, w, shared_out)
        mark(6)
        return out


def shard_experts(packed_w1: torch.Tensor, w2: torch.Tensor, rank: int, world: int):
    """Contiguous expert slice of rank `rank` (E/world experts)."""
    E = packed_w1.shape[0]
    El = E // world
    return packed_w1[rank * El:(rank + 1) * El], w2[rank * El:(rank + 1) * El]
