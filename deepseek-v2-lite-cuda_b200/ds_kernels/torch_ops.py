"""The drop-in ops as torch custom operators: `torch.ops.ds_kernels.<name>`.

The reference exposes its kernels as a pybind11 torch extension (src/kernels/bindings.cu:77-192),
so they are ordinary callables that torch.compile, torch.export and FakeTensor shape
propagation cannot see through.  Here every op of that surface is also registered with
`torch.library.custom_op` under the `ds_kernels` namespace, with a fake (meta) kernel that
gives the output shapes and dtypes from the input shapes alone:

    moe_routing  moe_scan  moe_dispatch  moe_combine  swiglu  moe_gemm1  moe_gemm2
    rms_norm  kv_upproj  rope
    (additive) moe_gemm1_swiglu  rms_norm_residual  moe_layer_fused

The real kernel of each operator is the eager function of the same name in `ds_kernels`
(the C-ABI call of libds_kernels_sm100.so through ctypes), so the two produce the same
bits.  Multi-output ops return tuples here (the operator schema's form) where the eager
functions return lists, as the reference binding does.  Inside torch.compile tracing the
eager functions route themselves through these operators (see `ds_kernels._traced`).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

import ds_kernels as _k

_NS = "ds_kernels"
Tensor = torch.Tensor


@torch.library.custom_op(f"{_NS}::moe_routing", mutates_args=())
def moe_routing(logits: Tensor, top_k: int = 6) -> Tuple[Tensor, Tensor, Tensor]:
    idx, w, counts = _k._eager["moe_routing"](logits, top_k)
    return idx, w, counts


@moe_routing.register_fake
def _(logits, top_k=6):
    T, E = logits.shape
    return (logits.new_empty((T, top_k), dtype=torch.int32),
            logits.new_empty((T, top_k), dtype=torch.float32),
            logits.new_empty((E,), dtype=torch.int32))


@torch.library.custom_op(f"{_NS}::moe_scan", mutates_args=())
def moe_scan(expert_counts: Tensor) -> Tensor:
    return _k._eager["moe_scan"](expert_counts)


@moe_scan.register_fake
def _(expert_counts):
    return expert_counts.new_empty((expert_counts.shape[0] + 1,), dtype=torch.int32)


@torch.library.custom_op(f"{_NS}::moe_dispatch", mutates_args=())
def moe_dispatch(input: Tensor, topk_indices: Tensor, topk_weights: Tensor,
                 expert_offsets: Tensor) -> Tuple[Tensor, Tensor, Tensor]:
    d, tm, dw = _k._eager["moe_dispatch"](input, topk_indices, topk_weights, expert_offsets)
    return d, tm, dw


@moe_dispatch.register_fake
def _(input, topk_indices, topk_weights, expert_offsets):
    S = topk_indices.shape[0] * topk_indices.shape[1]
    return (input.new_empty((S, input.shape[1]), dtype=torch.bfloat16),
            input.new_empty((S,), dtype=torch.int32),
            input.new_empty((S,), dtype=torch.float32))


@torch.library.custom_op(f"{_NS}::moe_combine", mutates_args=())
def moe_combine(expert_output: Tensor, token_map: Tensor, dispatched_weights: Tensor,
                num_tokens: int) -> Tensor:
    return _k._eager["moe_combine"](expert_output, token_map, dispatched_weights, num_tokens)


@moe_combine.register_fake
def _(expert_output, token_map, dispatched_weights, num_tokens):
    return expert_output.new_empty((num_tokens, expert_output.shape[1]), dtype=torch.bfloat16)


@torch.library.custom_op(f"{_NS}::swiglu", mutates_args=())
def swiglu(input: Tensor) -> Tensor:
    return _k._eager["swiglu"](input)


@swiglu.register_fake
def _(input):
    return input.new_empty((input.shape[0], input.shape[1] // 2), dtype=torch.bfloat16)


@torch.library.custom_op(f"{_NS}::moe_gemm1", mutates_args=())
def moe_gemm1(dispatched: Tensor, packed_w1: Tensor, expert_offsets: Tensor) -> Tensor:
    return _k._eager["moe_gemm1"](dispatched, packed_w1, expert_offsets)


@moe_gemm1.register_fake
def _(dispatched, packed_w1, expert_offsets):
    return dispatched.new_empty((dispatched.shape[0], packed_w1.shape[1]), dtype=torch.bfloat16)


@torch.library.custom_op(f"{_NS}::moe_gemm1_swiglu", mutates_args=())
def moe_gemm1_swiglu(dispatched: Tensor, packed_w1: Tensor, expert_offsets: Tensor) -> Tensor:
    return _k._eager["moe_gemm1_swiglu"](dispatched, packed_w1, expert_offsets)


@moe_gemm1_swiglu.register_fake
def _(dispatched, packed_w1, expert_offsets):
    return dispatched.new_empty((dispatched.shape[0], packed_w1.shape[1] // 2),
                                dtype=torch.bfloat16)


@torch.library.custom_op(f"{_NS}::moe_gemm2", mutates_args=())
def moe_gemm2(swiglu_out: Tensor, w2: Tensor, expert_offsets: Tensor) -> Tensor:
    return _k._eager["moe_gemm2"](swiglu_out, w2, expert_offsets)


@moe_gemm2.register_fake
def _(swiglu_out, w2, expert_offsets):
    return swiglu_out.new_empty((swiglu_out.shape[0], w2.shape[1]), dtype=torch.bfloat16)


@torch.library.custom_op(f"{_NS}::rms_norm", mutates_args=())
def rms_norm(input: Tensor, weight: Tensor, eps: float = 1e-6) -> Tensor:
    return _k._eager["rms_norm"](input, weight, eps)


@rms_norm.register_fake
def _(input, weight, eps=1e-6):
    return torch.empty_like(input)


@torch.library.custom_op(f"{_NS}::rms_norm_residual", mutates_args=())
def rms_norm_residual(input: Tensor, residual: Tensor, weight: Tensor,
                      eps: float = 1e-6) -> Tuple[Tensor, Tensor]:
    n, s = _k._eager["rms_norm_residual"](input, residual, weight, eps)
    return n, s


@rms_norm_residual.register_fake
def _(input, residual, weight, eps=1e-6):
    return torch.empty_like(input), torch.empty_like(input)


@torch.library.custom_op(f"{_NS}::kv_upproj", mutates_args=())
def kv_upproj(normed_kv: Tensor, weight: Tensor) -> Tensor:
    return _k._eager["kv_upproj"](normed_kv, weight)


@kv_upproj.register_fake
def _(normed_kv, weight):
    return normed_kv.new_empty((*normed_kv.shape[:-1], weight.shape[0]), dtype=torch.bfloat16)


@torch.library.custom_op(f"{_NS}::rope", mutates_args=())
def rope(q_pe: Tensor, k_pe: Tensor, cos: Tensor, sin: Tensor) -> Tuple[Tensor, Tensor]:
    q, k = _k._eager["rope"](q_pe, k_pe, cos, sin)
    return q, k


@rope.register_fake
def _(q_pe, k_pe, cos, sin):
    return torch.empty_like(q_pe), torch.empty_like(k_pe)


@torch.library.custom_op(f"{_NS}::moe_layer_fused", mutates_args=())
def moe_layer_fused(hidden_states: Tensor, gate_weight: Tensor, packed_w1: Tensor, w2: Tensor,
                    shared_w1: Optional[Tensor] = None, shared_w2: Optional[Tensor] = None,
                    top_k: int = 6) -> Tensor:
    return _k._eager["moe_layer_fused"](hidden_states, gate_weight, packed_w1, w2, shared_w1,
                                        shared_w2, top_k)


@moe_layer_fused.register_fake
def _(hidden_states, gate_weight, packed_w1, w2, shared_w1=None, shared_w2=None, top_k=6):
    return torch.empty_like(hidden_states)


OPS = ("moe_routing", "moe_scan", "moe_dispatch", "moe_combine", "swiglu", "moe_gemm1",
       "moe_gemm2", "rms_norm", "kv_upproj", "rope", "moe_gemm1_swiglu", "rms_norm_residual",
       "moe_layer_fused")
