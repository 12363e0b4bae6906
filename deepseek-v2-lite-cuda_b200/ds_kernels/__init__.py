"""ds_kernels — drop-in for the reference's `ds_kernels` extension module.

Same function names, argument names, defaults and return conventions as the reference
binding (src/kernels/bindings.cu:186-301): `moe_routing`, `moe_scan`, `moe_dispatch`,
`moe_combine`, `swiglu`, `moe_gemm1`, `moe_gemm2`, `rms_norm`, `kv_upproj`, `rope`,
`run_hello`; plus the additive ops `moe_gemm1_swiglu`, `moe_layer_fused` /
`moe_layer_forward` / `moe_layer_forward_from_x`, the layer stages and the expert-parallel
entry points.

Every op validates its tensors with the reference's messages (raising RuntimeError, as
TORCH_CHECK does), allocates outputs with torch on the input's device, and calls the
C ABI of libds_kernels_sm100.so (include/ds_kernels.h) through ctypes on the current torch
stream.  There is no fallback: if the library cannot be loaded, importing this module
raises ImportError, and every op requires CUDA tensors.
"""
from __future__ import annotations

import ctypes
import os
from typing import List, Optional, Sequence

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIBRARY_PATH = os.path.join(_HERE, "libds_kernels_sm100.so")

DS_OK = 0
DS_ERR_INVALID_ARG = 1
DS_ERR_UNSUPPORTED = 2
DS_ERR_CUDA = 3
DS_ERR_TIMEOUT = 4
DS_ERR_WORKSPACE = 5
LAYER_NUM_EVENTS = 9
MLA_NUM_EVENTS = 7
MLA_DECODE_NUM_EVENTS = 5
EP_NUM_EVENTS = 7
EP_IPC_HANDLE_BYTES = 64

_vp = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_sz = ctypes.c_size_t
_f = ctypes.c_float

# name -> (restype, argtypes); must match include/ds_kernels.h.
SIGNATURES = {
    "ds_last_error": (ctypes.c_char_p, []),
    "ds_version": (ctypes.c_char_p, []),
    "ds_get_device_status": (_i, [ctypes.POINTER(_i)]),
    "ds_clear_device_status": (_i, []),
    "ds_run_hello": (_i, [_vp]),
    "ds_moe_routing": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "ds_moe_scan": (_i, [_vp, _vp, _i, _vp]),
    "ds_moe_dispatch_workspace_size": (_sz, [_i, _i, _i]),
    "ds_moe_dispatch": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _sz, _vp]),
    "ds_moe_dispatch_noalloc": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "ds_moe_combine_workspace_size": (_sz, [_i, _i]),
    "ds_moe_combine": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _vp, _sz, _vp]),
    "ds_swiglu": (_i, [_vp, _vp, _i, _i, _vp]),
    "ds_moe_gemm1": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "ds_moe_gemm1_swiglu": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "ds_moe_gemm2": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "ds_rms_norm": (_i, [_vp, _vp, _vp, _i, _i, _f, _vp]),
    "ds_rms_norm_strided": (_i, [_vp, _i64, _vp, _vp, _i64, _i, _i, _f, _vp]),
    "ds_rms_norm_residual": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _f, _vp]),
    "ds_kv_upproj": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp]),
    "ds_gemm_pair_mode": (_i, [_i]),
    "ds_rope": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "ds_moe_layer_workspace_size": (_sz, [_i, _i, _i, _i, _i, _i]),
    "ds_mla_attention_workspace_size": (_sz, [_i, _i, _i]),
    "ds_mla_attention": (_i, [_vp, _i, _vp, _vp, _i, _i, _i, _f, _vp, _sz, _vp]),
    "ds_mla_forward_workspace_size": (_sz, [_i, _i, _i, _i]),
    "ds_mla_forward": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _f, _f,
                            _vp, _sz, _vp, _vp]),
    "ds_mla_prefill": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _f, _f, _vp,
                            _vp, _vp, _vp, _i, _i, _vp, _sz, _vp]),
    "ds_mla_cache_append": (_i, [_vp, _i, _vp, _i, _i, _i, _i, _i, _i, _i, _vp, _vp, _vp, _vp,
                                 _vp, _vp, _f, _vp]),
    "ds_mla_decode_workspace_size": (_sz, [_i, _i, _i]),
    "ds_mla_decode_step": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp, _i,
                                _i, _f, _f, _vp, _vp, _sz, _vp, _vp]),
    "ds_moe_layer_workspace_routing": (_i, [_i, _i, _i, _i, _i, _i, ctypes.POINTER(_sz),
                                            ctypes.POINTER(_sz), ctypes.POINTER(_sz)]),
    "ds_moe_layer_forward": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i,
                                  _vp, _sz, _vp, _vp]),
    "ds_debug_wait_probe": (_i, [ctypes.c_longlong, _vp]),
    "ds_moe_route_dispatch_workspace_size": (_sz, [_i, _i, _i]),
    "ds_moe_route_dispatch": (_i, [_vp, _vp, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                   _sz, _vp]),
    "ds_moe_expert_mlp": (_i, [_vp, _i, _vp, _i, _vp, _vp, _i, _i, _vp, _vp, _vp, _i, _vp]),
    "ds_dense_mlp": (_i, [_vp, _i, _vp, _vp, _i, _i, _vp, _vp, _i, _vp]),
    "ds_dense_mlp_workspace_size": (_sz, [_i, _i, _i]),
    "ds_dense_mlp_ws": (_i, [_vp, _i, _vp, _vp, _i, _i, _vp, _vp, _vp, _sz, _vp]),
    "ds_router_weight_split": (_i, [_vp, _i, _i, _vp, _vp]),
    "ds_dense_gemm1_swiglu": (_i, [_vp, _i, _vp, _i, _i, _vp, _i, _vp]),
    "ds_dense_gemm2": (_i, [_vp, _i, _vp, _i, _i, _vp, _i, _vp]),
    "ds_moe_router_workspace_size": (_sz, [_i]),
    "ds_moe_router": (_i, [_vp, _vp, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _sz, _vp]),
    "ds_moe_dispatch_routed": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _sz,
                                    _vp]),
    "ds_moe_layer_forward_from_x": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i,
                                         _i, _i, _vp, _sz, _vp, _vp]),
    "ds_moe_combine_slots": (_i, [_vp, _vp, _vp, _i, _vp, _vp, _i, _i, _vp]),
    "ds_ep_plan_workspace_size": (_sz, [_i, _i]),
    "ds_ep_plan": (_i, [_vp, _i, _i, _i, _vp, _vp, _vp, _sz, _vp]),
    "ds_gather_rows": (_i, [_vp, _vp, _i, _i, _vp, _vp]),
    "ds_ep_symmetric_size": (_i, [_i, _i, _i, _i, _i, ctypes.POINTER(_sz)]),
    "ds_ep_alloc": (_i, [_sz, ctypes.POINTER(_vp)]),
    "ds_ep_free": (_i, [_vp]),
    "ds_ep_ipc_handle": (_i, [_vp, _vp]),
    "ds_ep_ipc_open": (_i, [_vp, ctypes.POINTER(_vp)]),
    "ds_ep_ipc_close": (_i, [_vp]),
    "ds_ep_layer_workspace_size": (_sz, [_i, _i, _i, _i, _i, _i, _i]),
    "ds_ep_layer_forward": (_i, [_vp, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i,
                                 _i, _i, _i, _vp, _i, _i, _vp, _sz, _vp, _vp]),
}


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIBRARY_PATH):
        raise ImportError(
            f"ds_kernels: {LIBRARY_PATH} is missing; build it with "
            "`python deepseek-v2-lite-cuda_b200/build.py` (or __graft_entry__.build())")
    lib = ctypes.CDLL(LIBRARY_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_lib = _load()


def library() -> ctypes.CDLL:
    """The loaded libds_kernels_sm100.so handle (for direct C-ABI calls)."""
    return _lib


def version() -> str:
    return _lib.ds_version().decode()


def _check(status: int, op: str) -> None:
    if status != DS_OK:
        msg = _lib.ds_last_error().decode(errors="replace")
        raise RuntimeError(f"{op}: {msg} (status {status})")


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


class _on_device:
    """Make the tensor's device current for the duration of a C-ABI call."""

    def __init__(self, t: torch.Tensor):
        self.ctx = torch.cuda.device(t.device)

    def __enter__(self):
        self.ctx.__enter__()

    def __exit__(self, *exc):
        return self.ctx.__exit__(*exc)


# --------------------------------------------------------------------------------------------
def run_hello() -> None:
    """Executes the hello world CUDA kernel (toolchain smoke test)."""
    _check(_lib.ds_run_hello(torch.cuda.current_stream().cuda_stream), "run_hello")
    torch.cuda.synchronize()


def moe_routing(logits: torch.Tensor, top_k: int = 6) -> List[torch.Tensor]:
    """Fused softmax and top-K MoE routing kernel.

    Mirrors moe_routing_forward (src/kernels/moe/routing.cu:266-301).  Returns
    [topk_indices int32 [T, top_k], topk_weights float32 [T, top_k], expert_counts int32 [E]].
    Experts per token are ordered by descending logit, ties broken toward lower index.
    """
    _require(logits.is_cuda, "Input logits must reside on a CUDA device.")
    _require(logits.is_contiguous(), "Input logits must be contiguous in memory.")
    _require(logits.dtype == torch.float32, "Input logits must be of type float32.")
    _require(logits.dim() == 2, "Input logits must be a 2-D tensor [tokens, experts].")
    num_tokens, num_experts = logits.shape
    _require(num_experts <= 64, "num_experts must not exceed 64.")
    _require(1 <= top_k <= min(8, num_experts), "top_k must be in [1, min(8, num_experts)].")
    dev = logits.device
    idx = torch.empty((num_tokens, top_k), dtype=torch.int32, device=dev)
    w = torch.empty((num_tokens, top_k), dtype=torch.float32, device=dev)
    counts = torch.empty((num_experts,), dtype=torch.int32, device=dev)
    with _on_device(logits):
        _check(_lib.ds_moe_routing(_ptr(logits), _ptr(idx), _ptr(w), _ptr(counts), num_tokens,
                                   num_experts, top_k, _stream(logits)), "moe_routing")
    return [idx, w, counts]


def moe_scan(expert_counts: torch.Tensor) -> torch.Tensor:
    """Exclusive prefix sum of expert token counts -> expert_offsets int32 [E + 1].

    Mirrors moe_scan_forward (src/kernels/moe/scan.cu:86-130) without its host syncs.
    """
    _require(expert_counts.is_cuda, "Input expert_counts must reside on a CUDA device.")
    _require(expert_counts.is_contiguous(), "Input expert_counts must be contiguous in memory.")
    _require(expert_counts.dtype == torch.int32, "Input expert_counts must be of type int32.")
    _require(expert_counts.dim() == 1, "Input expert_counts must be a 1-D tensor [num_experts].")
    num_experts = expert_counts.shape[0]
    out = torch.empty((num_experts + 1,), dtype=torch.int32, device=expert_counts.device)
    if num_experts == 0:
        out.zero_()
        return out
    with _on_device(expert_counts):
        _check(_lib.ds_moe_scan(_ptr(expert_counts), _ptr(out), num_experts,
                                _stream(expert_counts)), "moe_scan")
    return out


def _check_tensor(t: torch.Tensor, name: str, dtype: torch.dtype, dtype_name: str, dim: int,
                  shape_doc: str) -> None:
    _require(t.is_cuda, f"{name} must reside on a CUDA device.")
    _require(t.is_contiguous(), f"{name} must be contiguous in memory.")
    _require(t.dtype == dtype, f"{name} must be of type {dtype_name}.")
    _require(t.dim() == dim, f"{name} must be a {dim}-D tensor {shape_doc}.")


def moe_dispatch(input: torch.Tensor, topk_indices: torch.Tensor, topk_weights: torch.Tensor,
                 expert_offsets: torch.Tensor) -> List[torch.Tensor]:
    """Scatters token hidden states into an expert-contiguous output buffer.

    Mirrors moe_dispatch_forward (src/kernels/moe/dispatch.cu:156-218).  Returns
    [dispatched bf16 [T*k, H], token_map int32 [T*k], dispatched_weights float32 [T*k]].
    Slots inside an expert hold its tokens in ascending token order.
    """
    _check_tensor(input, "input", torch.bfloat16, "bfloat16", 2, "[num_tokens, hidden_size]")
    _check_tensor(topk_indices, "topk_indices", torch.int32, "int32", 2, "[num_tokens, top_k]")
    _check_tensor(topk_weights, "topk_weights", torch.float32, "float32", 2,
                  "[num_tokens, top_k]")
    _check_tensor(expert_offsets, "expert_offsets", torch.int32, "int32", 1,
                  "[num_experts + 1]")
    num_tokens, hidden = input.shape
    top_k = topk_indices.shape[1]
    num_experts = expert_offsets.shape[0] - 1
    _require(hidden % 8 == 0, "hidden_size must be divisible by 8 for 128-bit vectorized access.")
    total = num_tokens * top_k
    dev = input.device
    dispatched = torch.empty((total, hidden), dtype=torch.bfloat16, device=dev)
    token_map = torch.empty((total,), dtype=torch.int32, device=dev)
    dweights = torch.empty((total,), dtype=torch.float32, device=dev)
    if total == 0:
        return [dispatched, token_map, dweights]
    ws_bytes = _lib.ds_moe_dispatch_workspace_size(num_tokens, num_experts, top_k)
    ws = _workspace(ws_bytes, dev)
    with _on_device(input):
        _check(_lib.ds_moe_dispatch(_ptr(input), _ptr(topk_indices), _ptr(topk_weights),
                                    _ptr(expert_offsets), _ptr(dispatched), _ptr(token_map),
                                    _ptr(dweights), num_tokens, hidden, num_experts, top_k,
                                    _ptr(ws), ws_bytes, _stream(input)), "moe_dispatch")
    return [dispatched, token_map, dweights]


def moe_combine(expert_output: torch.Tensor, token_map: torch.Tensor,
                dispatched_weights: torch.Tensor, num_tokens: int) -> torch.Tensor:
    """Accumulates weighted expert outputs back to token-ordered positions.

    Mirrors moe_combine_forward (src/kernels/moe/combine.cu:107-176): f32 accumulation,
    one bf16 rounding; token_map may hold any multiplicity.  Deterministic.
    """
    _check_tensor(expert_output, "expert_output", torch.bfloat16, "bfloat16", 2,
                  "[total_slots, hidden_size]")
    _check_tensor(token_map, "token_map", torch.int32, "int32", 1, "[total_slots]")
    _check_tensor(dispatched_weights, "dispatched_weights", torch.float32, "float32", 1,
                  "[total_slots]")
    _require(num_tokens > 0, "num_tokens must be positive.")
    total, hidden = expert_output.shape
    dev = expert_output.device
    out = torch.empty((num_tokens, hidden), dtype=torch.bfloat16, device=dev)
    ws_bytes = _lib.ds_moe_combine_workspace_size(total, num_tokens)
    ws = _workspace(ws_bytes, dev)
    with _on_device(expert_output):
        _check(_lib.ds_moe_combine(_ptr(expert_output), _ptr(token_map),
                                   _ptr(dispatched_weights), _ptr(out), total, hidden,
                                   num_tokens, _ptr(ws), ws_bytes, _stream(expert_output)),
               "moe_combine")
    return out


def swiglu(input: torch.Tensor) -> torch.Tensor:
    """SwiGLU activation: silu(gate_half) * up_half  ([S, 2I] bf16 -> [S, I] bf16).

    Mirrors swiglu_forward (src/kernels/moe/swiglu.cu:142-170).
    """
    _require(input.is_cuda, "swiglu: input must be a CUDA tensor.")
    _require(input.is_contiguous(), "swiglu: input must be contiguous.")
    _require(input.dtype == torch.bfloat16, "swiglu: input must be bfloat16.")
    _require(input.dim() == 2, "swiglu: input must be 2-D [total_tokens, 2*intermediate_size].")
    _require(input.shape[1] % 2 == 0, "swiglu: input inner dimension must be even.")
    rows, two_i = input.shape
    inter = two_i // 2
    out = torch.empty((rows, inter), dtype=torch.bfloat16, device=input.device)
    if rows == 0:
        return out
    with _on_device(input):
        _check(_lib.ds_swiglu(_ptr(input), _ptr(out), rows, inter, _stream(input)), "swiglu")
    return out


def _gemm_checks(a: torch.Tensor, w: torch.Tensor, off: torch.Tensor, tag: str,
                 a_doc: str, w_doc: str) -> None:
    _require(a.is_cuda and a.is_contiguous(), f"{tag}: {a_doc} must be a contiguous CUDA tensor.")
    _require(a.dtype == torch.bfloat16, f"{tag}: {a_doc} must be bfloat16.")
    _require(a.dim() == 2, f"{tag}: {a_doc} must be 2-D [total_slots, hidden_size].")
    _require(w.is_cuda and w.is_contiguous(), f"{tag}: {w_doc} must be a contiguous CUDA tensor.")
    _require(w.dtype == torch.bfloat16, f"{tag}: {w_doc} must be bfloat16.")
    _require(w.dim() == 3, f"{tag}: {w_doc} must be 3-D.")
    _require(off.is_cuda and off.is_contiguous(),
             f"{tag}: expert_offsets must be a contiguous CUDA tensor.")
    _require(off.dtype == torch.int32, f"{tag}: expert_offsets must be int32.")
    _require(off.dim() == 1, f"{tag}: expert_offsets must be 1-D [num_experts + 1].")
    _require(off.shape[0] == w.shape[0] + 1, f"{tag}: expert_offsets size must be num_experts + 1.")


def _moe_gemm1(dispatched, packed_w1, expert_offsets, fused: bool) -> torch.Tensor:
    _gemm_checks(dispatched, packed_w1, expert_offsets, "gemm1", "dispatched", "packed_w1")
    total, hidden = dispatched.shape
    num_experts, two_i, _ = packed_w1.shape
    _require(packed_w1.shape[2] == hidden,
             "gemm1: packed_w1 hidden_size dim does not match dispatched.")
    cols = two_i // 2 if fused else two_i
    out = torch.empty((total, cols), dtype=torch.bfloat16, device=dispatched.device)
    if total == 0:
        return out
    fn = _lib.ds_moe_gemm1_swiglu if fused else _lib.ds_moe_gemm1
    with _on_device(dispatched):
        _check(fn(_ptr(dispatched), _ptr(packed_w1), _ptr(expert_offsets), _ptr(out), total,
                  num_experts, hidden, two_i, _stream(dispatched)),
               "moe_gemm1_swiglu" if fused else "moe_gemm1")
    return out


def moe_gemm1(dispatched: torch.Tensor, packed_w1: torch.Tensor,
              expert_offsets: torch.Tensor) -> torch.Tensor:
    """Batched gate+up projection for all active experts (tcgen05 grouped GEMM).

    Mirrors moe_gemm1_forward (src/kernels/moe/gemm1.cu:167-227); offsets stay on device.
    """
    return _moe_gemm1(dispatched, packed_w1, expert_offsets, fused=False)


def moe_gemm1_swiglu(dispatched: torch.Tensor, packed_w1: torch.Tensor,
                     expert_offsets: torch.Tensor) -> torch.Tensor:
    """GEMM1 with the SwiGLU epilogue fused: [S, H] -> [S, I] (new, additive op)."""
    return _moe_gemm1(dispatched, packed_w1, expert_offsets, fused=True)


def moe_gemm2(swiglu_out: torch.Tensor, w2: torch.Tensor,
              expert_offsets: torch.Tensor) -> torch.Tensor:
    """Batched down_proj for all active experts (tcgen05 grouped GEMM).

    Mirrors moe_gemm2_forward (src/kernels/moe/gemm2.cu:136-195).
    """
    _gemm_checks(swiglu_out, w2, expert_offsets, "gemm2", "swiglu_out", "w2")
    total, inter = swiglu_out.shape
    num_experts, hidden, _ = w2.shape
    _require(w2.shape[2] == inter, "gemm2: w2 intermediate dim does not match swiglu_out.")
    out = torch.empty((total, hidden), dtype=torch.bfloat16, device=swiglu_out.device)
    if total == 0:
        return out
    with _on_device(swiglu_out):
        _check(_lib.ds_moe_gemm2(_ptr(swiglu_out), _ptr(w2), _ptr(expert_offsets), _ptr(out),
                                 total, num_experts, inter, hidden, _stream(swiglu_out)),
               "moe_gemm2")
    return out


def rms_norm(input: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """RMSNorm over the last dimension of a BF16 tensor (f32 weight).

    Mirrors rms_norm_forward (src/kernels/mla/rms_norm.cu:158-192).
    """
    _require(input.is_cuda, "rms_norm: input must be a CUDA tensor.")
    _require(weight.is_cuda, "rms_norm: weight must be a CUDA tensor.")
    _require(input.is_contiguous(), "rms_norm: input must be contiguous.")
    _require(input.dtype == torch.bfloat16, "rms_norm: input must be bfloat16.")
    _require(weight.dtype == torch.float32,
             "rms_norm: weight must be float32 (default nn.Parameter dtype).")
    _require(input.dim() >= 2, "rms_norm: input must have at least 2 dimensions.")
    hidden = input.shape[-1]
    _require(weight.numel() == hidden,
             f"rms_norm: weight size {weight.numel()} does not match input hidden_size {hidden}.")
    _require(hidden % 2 == 0, "rms_norm: hidden_size must be even for bfloat162 vectorisation.")
    weight = weight.contiguous()
    rows = input.numel() // hidden if hidden else 0
    out = torch.empty_like(input)
    if rows == 0:
        return out
    with _on_device(input):
        _check(_lib.ds_rms_norm(_ptr(input), _ptr(weight), _ptr(out), rows, hidden, float(eps),
                                _stream(input)), "rms_norm")
    return out


def rms_norm_residual(input: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                      eps: float = 1e-6) -> List[torch.Tensor]:
    """Decoder-layer glue: returns [normed, sum] with sum = bf16(residual + input) (the next
    residual) and normed = RMSNorm(sum) — the residual add and pre-norm around the attention
    and MoE sub-layers of src/reference/decoder_layer.py:123-139, in one pass."""
    _require(input.is_cuda and residual.is_cuda and weight.is_cuda,
             "rms_norm_residual: all inputs must be CUDA tensors.")
    _require(input.is_contiguous() and residual.is_contiguous(),
             "rms_norm_residual: input and residual must be contiguous.")
    _require(input.dtype == torch.bfloat16 and residual.dtype == torch.bfloat16,
             "rms_norm_residual: input and residual must be bfloat16.")
    _require(weight.dtype == torch.float32, "rms_norm_residual: weight must be float32.")
    _require(tuple(input.shape) == tuple(residual.shape) and input.dim() >= 1,
             "rms_norm_residual: input and residual must have the same shape.")
    H = input.shape[-1]
    _require(weight.numel() == H, "rms_norm_residual: weight size must match hidden_size.")
    rows = input.numel() // H if H else 0
    s = torch.empty_like(input)
    n = torch.empty_like(input)
    with _on_device(input):
        _check(_lib.ds_rms_norm_residual(_ptr(input), _ptr(residual), _ptr(weight.contiguous()),
                                         _ptr(s), _ptr(n), rows, H, float(eps), _stream(input)),
               "rms_norm_residual")
    return [n, s]


def gemm_pair_mode(mode: Optional[int] = None) -> int:
    """Tiling of the tcgen05 grouped GEMM (process-wide): 0 single-CTA 128x256 tiles, 1 CTA
    pairs on 256x256 tiles, -1 automatic; None only queries.  Returns the previous mode."""
    return _lib.ds_gemm_pair_mode(-2 if mode is None else int(mode))


def kv_upproj(normed_kv: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """KV up-projection: normed_kv @ kv_b_proj.weight.T (tcgen05 GEMM), keeps leading dims.

    Mirrors kv_upproj_forward (src/kernels/mla/kv_upproj.cu:133-178).
    """
    _require(normed_kv.is_cuda and normed_kv.is_contiguous(),
             "kv_upproj: normed_kv must be a contiguous CUDA tensor.")
    _require(normed_kv.dtype == torch.bfloat16, "kv_upproj: normed_kv must be bfloat16.")
    _require(normed_kv.dim() >= 2, "kv_upproj: normed_kv must have at least 2 dimensions.")
    _require(weight.is_cuda and weight.is_contiguous(),
             "kv_upproj: weight must be a contiguous CUDA tensor.")
    _require(weight.dtype == torch.bfloat16, "kv_upproj: weight must be bfloat16.")
    _require(weight.dim() == 2, "kv_upproj: weight must be 2-D [out_dim, kv_lora_rank].")
    rank = normed_kv.shape[-1]
    out_dim = weight.shape[0]
    _require(weight.shape[1] == rank,
             f"kv_upproj: weight inner dim {weight.shape[1]} must match normed_kv last dim {rank}.")
    rows = normed_kv.numel() // rank if rank else 0
    out = torch.empty((*normed_kv.shape[:-1], out_dim), dtype=torch.bfloat16,
                      device=normed_kv.device)
    if rows == 0:
        return out
    with _on_device(normed_kv):
        _check(_lib.ds_kv_upproj(_ptr(normed_kv), _ptr(weight), _ptr(out), rows, rank, out_dim,
                                 _stream(normed_kv)), "kv_upproj")
    return out


def rope(q_pe: torch.Tensor, k_pe: torch.Tensor, cos: torch.Tensor,
         sin: torch.Tensor) -> List[torch.Tensor]:
    """YaRN RoPE applied to q_pe and k_pe (interleave->half transform + rotation).

    Mirrors rope_forward (src/kernels/mla/rope.cu:139-207) in a single launch; cos/sin are
    broadcast over heads by index instead of being expanded.  Returns [q_rot, k_rot].
    Strided inputs (e.g. the q_pe slice of the q projection) are accepted and made
    contiguous first; the reference rejects them.
    """
    for t in (q_pe, k_pe, cos, sin):
        _require(t.is_cuda, "rope: all inputs must be contiguous CUDA tensors.")
        _require(t.dtype == torch.bfloat16, "rope: all inputs must be bfloat16.")
    q_pe, k_pe, cos, sin = (t.contiguous() for t in (q_pe, k_pe, cos, sin))
    _require(q_pe.dim() == 4, "rope: q_pe must be 4-D [bsz, heads, seq, rope_dim].")
    _require(k_pe.dim() == 4, "rope: k_pe must be 4-D [bsz, 1, seq, rope_dim].")
    _require(cos.dim() == 4, "rope: cos must be 4-D [bsz, 1, seq, rope_dim].")
    _require(sin.dim() == 4, "rope: sin must be 4-D [bsz, 1, seq, rope_dim].")
    bsz, heads, seq, rope_dim = q_pe.shape
    _require(k_pe.shape[0] == bsz and k_pe.shape[1] == 1 and k_pe.shape[2] == seq
             and k_pe.shape[3] == rope_dim,
             f"rope: k_pe shape {list(k_pe.shape)} incompatible with q_pe.")
    _require(cos.shape[0] == bsz and cos.shape[1] == 1 and cos.shape[2] == seq
             and cos.shape[3] == rope_dim, "rope: cos shape incompatible.")
    _require(sin.shape[0] == bsz and sin.shape[1] == 1 and sin.shape[2] == seq
             and sin.shape[3] == rope_dim, "rope: sin shape incompatible.")
    _require(rope_dim % 2 == 0, "rope: rope_dim must be even.")
    q_rot = torch.empty_like(q_pe)
    k_rot = torch.empty_like(k_pe)
    if q_pe.numel() + k_pe.numel() == 0:
        return [q_rot, k_rot]
    with _on_device(q_pe):
        _check(_lib.ds_rope(_ptr(q_pe), _ptr(k_pe), _ptr(cos), _ptr(sin), _ptr(q_rot),
                            _ptr(k_rot), bsz, heads, seq, rope_dim, _stream(q_pe)), "rope")
    return [q_rot, k_rot]


def moe_layer_workspace_size(num_tokens: int, hidden_size: int, num_experts: int, top_k: int,
                             intermediate_size: int, shared_intermediate_size: int) -> int:
    return int(_lib.ds_moe_layer_workspace_size(num_tokens, hidden_size, num_experts, top_k,
                                                intermediate_size, shared_intermediate_size))


def moe_layer_workspace_routing(workspace: torch.Tensor, num_tokens: int, hidden_size: int,
                                num_experts: int, top_k: int, intermediate_size: int,
                                shared_intermediate_size: int):
    """Views of the routing a layer forward left in `workspace`: (topk_indices int32 [T, k],
    topk_weights f32 [T, k], slot_of int32 [T, k]); valid until the workspace is reused."""
    a, b, c = _sz(0), _sz(0), _sz(0)
    _check(_lib.ds_moe_layer_workspace_routing(num_tokens, hidden_size, num_experts, top_k,
                                               intermediate_size, shared_intermediate_size,
                                               ctypes.byref(a), ctypes.byref(b),
                                               ctypes.byref(c)), "moe_layer_workspace_routing")
    n = num_tokens * top_k

    def view(off, dtype):
        return workspace[off:off + 4 * n].view(dtype).view(num_tokens, top_k)
    return view(a.value, torch.int32), view(b.value, torch.float32), view(c.value, torch.int32)


def moe_layer_forward(router_logits: torch.Tensor, x: torch.Tensor, packed_w1: torch.Tensor,
                      w2: torch.Tensor, shared_w1: Optional[torch.Tensor] = None,
                      shared_w2: Optional[torch.Tensor] = None, top_k: int = 6,
                      out: Optional[torch.Tensor] = None,
                      workspace: Optional[torch.Tensor] = None,
                      events: Optional[Sequence[torch.cuda.Event]] = None) -> torch.Tensor:
    """Whole MoE layer in one C call (new, additive): routing -> dispatch -> grouped GEMMs
    (+ shared expert) -> combine.  router_logits f32 [T, E], x bf16 [T, H], packed_w1 bf16
    [E, 2I, H], w2 bf16 [E, H, I], shared_w1 bf16 [2Is, H] (gate rows then up rows),
    shared_w2 bf16 [H, Is].  `events` (9 torch.cuda.Event) are recorded between phases.
    """
    _check_tensor(router_logits, "router_logits", torch.float32, "float32", 2, "[T, E]")
    _check_tensor(x, "x", torch.bfloat16, "bfloat16", 2, "[T, H]")
    _require(packed_w1.is_contiguous() and packed_w1.dtype == torch.bfloat16 and packed_w1.dim() == 3,
             "packed_w1 must be a contiguous bf16 [E, 2I, H] tensor.")
    _require(w2.is_contiguous() and w2.dtype == torch.bfloat16 and w2.dim() == 3,
             "w2 must be a contiguous bf16 [E, H, I] tensor.")
    T, H = x.shape
    E = packed_w1.shape[0]
    I = packed_w1.shape[1] // 2
    _require(router_logits.shape == (T, E), "router_logits must be [T, num_experts].")
    _require(w2.shape == (E, H, I), "w2 must be [E, H, I].")
    Is = 0
    if shared_w1 is not None or shared_w2 is not None:
        _require(shared_w1 is not None and shared_w2 is not None,
                 "give both shared expert weights or neither")
        _require(shared_w1.is_contiguous() and shared_w1.dtype == torch.bfloat16
                 and shared_w1.dim() == 2 and shared_w1.shape[1] == H,
                 "shared_w1 must be a contiguous bf16 [2Is, H] tensor.")
        Is = shared_w1.shape[0] // 2
        _require(shared_w2.is_contiguous() and shared_w2.dtype == torch.bfloat16
                 and tuple(shared_w2.shape) == (H, Is),
                 "shared_w2 must be a contiguous bf16 [H, Is] tensor.")
    if out is None:
        out = torch.empty((T, H), dtype=torch.bfloat16, device=x.device)
    if T == 0:
        return out
    need = moe_layer_workspace_size(T, H, E, top_k, I, Is)
    if workspace is None or workspace.numel() < need:
        workspace = _workspace(need, x.device)
    ev = None
    if events is not None:
        _require(len(events) == LAYER_NUM_EVENTS, f"events must hold {LAYER_NUM_EVENTS} events")
        st = torch.cuda.current_stream(x.device)
        for e in events:  # torch creates events lazily; a record makes the handle valid
            e.record(st)
        ev = (ctypes.c_void_p * LAYER_NUM_EVENTS)(*[e.cuda_event for e in events])
    with _on_device(x):
        _check(_lib.ds_moe_layer_forward(_ptr(router_logits), _ptr(x), _ptr(packed_w1), _ptr(w2),
                                         _ptr(shared_w1), _ptr(shared_w2), _ptr(out), T, H, E,
                                         top_k, I, Is, _ptr(workspace), workspace.numel(), ev,
                                         _stream(x)), "moe_layer_forward")
    return out


def mla_attention(qkv: torch.Tensor, kv: torch.Tensor, batch: int, seq: int, heads: int,
                  softmax_scale: float, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Causal MLA attention core (src/reference/mla.py:355-378) on the tcgen05 tensor cores.

    qkv bf16 [batch*seq, ld]: per token the heads' q (192 each: 128 nope, then 64 already
    RoPE-rotated), the 512-wide latent, then the rotated 64-wide k_pe; kv bf16
    [batch*seq, heads*256]: per head 128 k_nope then 128 v.  Returns bf16
    [batch*seq, heads*128] (head h in columns h*128 ..)."""
    _check_tensor(qkv, "qkv", torch.bfloat16, "bfloat16", 2, "[batch*seq, ld]")
    _check_tensor(kv, "kv", torch.bfloat16, "bfloat16", 2, "[batch*seq, heads*256]")
    _require(qkv.shape[0] == batch * seq and kv.shape[0] == batch * seq,
             "mla_attention: qkv and kv must hold batch*seq rows")
    _require(kv.shape[1] == heads * 256, "mla_attention: kv must be [batch*seq, heads*256]")
    if out is None:
        out = torch.empty((batch * seq, heads * 128), dtype=torch.bfloat16, device=qkv.device)
    if batch * seq == 0:
        return out
    need = int(_lib.ds_mla_attention_workspace_size(batch, seq, heads))
    ws = _workspace(need, qkv.device)
    with _on_device(qkv):
        _check(_lib.ds_mla_attention(_ptr(qkv), qkv.shape[1], _ptr(kv), _ptr(out), batch, seq,
                                     heads, float(softmax_scale), _ptr(ws), need, _stream(qkv)),
               "mla_attention")
    return out


def mla_forward_workspace_size(batch: int, seq: int, hidden: int, heads: int) -> int:
    return int(_lib.ds_mla_forward_workspace_size(batch, seq, hidden, heads))


def mla_forward(hidden_states: torch.Tensor, w_qkv_a: torch.Tensor,
                kv_norm_weight: torch.Tensor, w_kv_b: torch.Tensor, w_o: torch.Tensor,
                cos: torch.Tensor, sin: torch.Tensor, softmax_scale: float, heads: int,
                position_ids: Optional[torch.Tensor] = None, eps: float = 1e-6,
                workspace: Optional[torch.Tensor] = None,
                events: Optional[Sequence[torch.cuda.Event]] = None) -> torch.Tensor:
    """The whole MLA forward of DeepSeekMLA (src/reference/mla.py:295-393) in one C call:
    hidden_states bf16 [batch, seq, hidden] -> bf16 [batch, seq, hidden].  w_qkv_a =
    cat(q_proj.weight, kv_a_proj_with_mqa.weight) bf16 [heads*192 + 576, hidden];
    kv_norm_weight f32 [512]; w_kv_b bf16 [heads*256, 512]; w_o bf16 [hidden, heads*128];
    cos/sin bf16 [positions, 64]; position_ids int [batch, seq] or None (0..seq-1)."""
    _require(hidden_states.is_cuda and hidden_states.dtype == torch.bfloat16
             and hidden_states.dim() == 3, "mla_forward: hidden_states must be CUDA bf16 [b, s, h]")
    x = hidden_states.contiguous()
    B, S, Hd = x.shape
    for t, name in ((w_qkv_a, "w_qkv_a"), (w_kv_b, "w_kv_b"), (w_o, "w_o"), (cos, "cos"),
                    (sin, "sin")):
        _require(t.is_cuda and t.is_contiguous() and t.dtype == torch.bfloat16,
                 f"mla_forward: {name} must be a contiguous CUDA bf16 tensor")
    _require(tuple(w_qkv_a.shape) == (heads * 192 + 576, Hd), "mla_forward: w_qkv_a shape")
    _require(tuple(w_kv_b.shape) == (heads * 256, 512), "mla_forward: w_kv_b shape")
    _require(tuple(w_o.shape) == (Hd, heads * 128), "mla_forward: w_o shape")
    _require(cos.dim() == 2 and cos.shape[1] == 64 and tuple(sin.shape) == tuple(cos.shape),
             "mla_forward: cos/sin must be [positions, 64]")
    nw = kv_norm_weight.detach().float().contiguous()
    pos = None
    if position_ids is not None:
        pos = position_ids.to(device=x.device, dtype=torch.int32).expand(B, S).contiguous()
        _require(int(pos.max()) < cos.shape[0] and int(pos.min()) >= 0,
                 "mla_forward: position_ids outside the cos/sin tables")
    else:
        _require(S <= cos.shape[0], "mla_forward: seq_len exceeds the cos/sin tables")
    out = torch.empty((B, S, Hd), dtype=torch.bfloat16, device=x.device)
    if B * S == 0:
        return out
    need = mla_forward_workspace_size(B, S, Hd, heads)
    if workspace is None or workspace.numel() < need:
        workspace = _workspace(need, x.device)
    ev = None
    if events is not None:
        _require(len(events) == MLA_NUM_EVENTS, f"events must hold {MLA_NUM_EVENTS} events")
        st = torch.cuda.current_stream(x.device)
        for e in events:
            e.record(st)
        ev = (ctypes.c_void_p * MLA_NUM_EVENTS)(*[e.cuda_event for e in events])
    with _on_device(x):
        _check(_lib.ds_mla_forward(_ptr(x), _ptr(w_qkv_a), _ptr(nw), _ptr(w_kv_b), _ptr(w_o),
                                   _ptr(cos), _ptr(sin), _ptr(pos), _ptr(out), B, S, Hd, heads,
                                   float(eps), float(softmax_scale), _ptr(workspace),
                                   workspace.numel(), ev, _stream(x)), "mla_forward")
    return out


def mla_prefill(hidden_states: torch.Tensor, w_qkv_a: torch.Tensor,
                kv_norm_weight: torch.Tensor, w_kv_b: torch.Tensor, w_o: torch.Tensor,
                cos: torch.Tensor, sin: torch.Tensor, softmax_scale: float, heads: int, cache,
                eps: float = 1e-6, workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """mla_forward over a prompt at positions 0 .. seq-1 that also fills `cache` (an empty
    mla_cache.LatentKVCache on the same device) with the prompt's raw latents and k_pe."""
    x = hidden_states.contiguous()
    B, S, Hd = x.shape
    _require(cache.current_len == 0, "mla_prefill: the cache must be empty")
    _require(cache.bsz == B and S <= cache.max_seq, "mla_prefill: cache shape")
    out = torch.empty((B, S, Hd), dtype=torch.bfloat16, device=x.device)
    if B * S == 0:
        return out
    need = mla_forward_workspace_size(B, S, Hd, heads)
    if workspace is None or workspace.numel() < need:
        workspace = _workspace(need, x.device)
    nw = kv_norm_weight.detach().float().contiguous()
    with _on_device(x):
        _check(_lib.ds_mla_prefill(_ptr(x), _ptr(w_qkv_a), _ptr(nw), _ptr(w_kv_b), _ptr(w_o),
                                   _ptr(cos), _ptr(sin), _ptr(out), B, S, Hd, heads, float(eps),
                                   float(softmax_scale), _ptr(cache.kv_latent),
                                   _ptr(cache.k_pe_cache), _ptr(cache.rstd), _ptr(cache.k_pe_rot),
                                   cache.max_seq, 0, _ptr(workspace), workspace.numel(),
                                   _stream(x)), "mla_prefill")
    cache._advance(S, device_counted=False)
    return out


def mla_cache_append(latent: torch.Tensor, k_pe: torch.Tensor, cache, pos0: int,
                     cos: torch.Tensor, sin: torch.Tensor, eps: float = 1e-6,
                     copy_raw: bool = True) -> None:
    """latent [bsz, n, 512], k_pe [bsz, n, 64] (bf16, CUDA; any row stride with 16-byte aligned
    rows) -> cache positions pos0 .. pos0+n-1, with the side arrays (rstd, rotated k_pe)."""
    B, n, _ = latent.shape
    if B * n == 0:
        return
    _require(latent.stride(2) == 1 and k_pe.stride(2) == 1, "mla_cache_append: unsupported strides")
    rows = latent.stride(0) // latent.stride(1)
    _require(latent.stride(0) == rows * latent.stride(1)
             and k_pe.stride(0) == rows * k_pe.stride(1),
             "mla_cache_append: latent and k_pe must step sequences by the same number of rows")
    with _on_device(latent):
        _check(_lib.ds_mla_cache_append(_ptr(latent), latent.stride(1), _ptr(k_pe), k_pe.stride(1),
                                        rows, B, n, pos0, cache.max_seq, 1 if copy_raw else 0,
                                        _ptr(cache.kv_latent), _ptr(cache.k_pe_cache),
                                        _ptr(cache.rstd), _ptr(cache.k_pe_rot), _ptr(cos),
                                        _ptr(sin), float(eps), _stream(latent)),
               "mla_cache_append")


def mla_decode_workspace_size(batch: int, max_seq: int, hidden: int) -> int:
    return int(_lib.ds_mla_decode_workspace_size(batch, max_seq, hidden))


def mla_decode_step(x: torch.Tensor, w_dec: torch.Tensor, w_out: torch.Tensor, cos: torch.Tensor,
                    sin: torch.Tensor, cache, softmax_scale: float, heads: int = 16,
                    eps: float = 1e-6, workspace: Optional[torch.Tensor] = None,
                    events: Optional[Sequence[torch.cuda.Event]] = None) -> torch.Tensor:
    """One decode step: x bf16 [bsz, hidden] (one new token per sequence) -> [bsz, hidden];
    appends the token to `cache` (mla_cache.LatentKVCache) at position cache.current_len and
    attends over every cached position (see include/ds_kernels.h for w_dec / w_out)."""
    _check_tensor(x, "x", torch.bfloat16, "bfloat16", 2, "[bsz, hidden]")
    B, Hd = x.shape
    _require(cache.bsz == B, "mla_decode_step: cache batch size differs from x")
    out = torch.empty((B, Hd), dtype=torch.bfloat16, device=x.device)
    need = mla_decode_workspace_size(B, cache.max_seq, Hd)
    if workspace is None or workspace.numel() < need:
        workspace = _workspace(need, x.device)
    ev = None
    if events is not None:
        _require(len(events) == MLA_DECODE_NUM_EVENTS,
                 f"events must hold {MLA_DECODE_NUM_EVENTS} events")
        st = torch.cuda.current_stream(x.device)
        for e in events:
            e.record(st)
        ev = (ctypes.c_void_p * MLA_DECODE_NUM_EVENTS)(*[e.cuda_event for e in events])
    cache._sync_side(cos, sin, eps)
    with _on_device(x):
        _check(_lib.ds_mla_decode_step(_ptr(x), _ptr(w_dec), _ptr(w_out), _ptr(cos), _ptr(sin),
                                       _ptr(cache.kv_latent), _ptr(cache.k_pe_cache),
                                       _ptr(cache.rstd), _ptr(cache.k_pe_rot), B, cache.max_seq,
                                       cache.current_len, _ptr(cache.len_dev), Hd, heads, float(eps),
                                       float(softmax_scale), _ptr(out), _ptr(workspace),
                                       workspace.numel(), ev, _stream(x)), "mla_decode_step")
    cache._advance(1, device_counted=True)
    return out


def device_status() -> int:
    """DS_OK or DS_ERR_TIMEOUT (set when an on-device bounded wait ran out). Synchronises."""
    v = ctypes.c_int(0)
    _check(_lib.ds_get_device_status(ctypes.byref(v)), "device_status")
    return v.value


def clear_device_status() -> None:
    _check(_lib.ds_clear_device_status(), "clear_device_status")


def debug_wait_probe(timeout_cycles: int) -> None:
    """Launch the bounded-wait probe (a wait nothing completes); see include/ds_kernels.h."""
    _check(_lib.ds_debug_wait_probe(int(timeout_cycles), torch.cuda.current_stream().cuda_stream),
           "debug_wait_probe")


# ---------------------------------------------------------------------------------- stages
def moe_route_dispatch(router_logits: torch.Tensor, x: torch.Tensor, top_k: int = 6):
    """Routing + offsets + deterministic dispatch in one call.

    Returns (topk_indices [T,k] i32, topk_weights [T,k] f32, expert_offsets [E+1] i32,
    slot_of [T,k] i32, token_map [T*k] i32, dispatched [T*k, H] bf16)."""
    _check_tensor(router_logits, "router_logits", torch.float32, "float32", 2, "[T, E]")
    _check_tensor(x, "x", torch.bfloat16, "bfloat16", 2, "[T, H]")
    T, H = x.shape
    E = router_logits.shape[1]
    dev = x.device
    idx = torch.empty((T, top_k), dtype=torch.int32, device=dev)
    w = torch.empty((T, top_k), dtype=torch.float32, device=dev)
    off = torch.empty((E + 1,), dtype=torch.int32, device=dev)
    slot_of = torch.empty((T, top_k), dtype=torch.int32, device=dev)
    tmap = torch.empty((T * top_k,), dtype=torch.int32, device=dev)
    disp = torch.empty((T * top_k, H), dtype=torch.bfloat16, device=dev)
    need = _lib.ds_moe_route_dispatch_workspace_size(T, E, top_k)
    ws = _workspace(need, dev)
    with _on_device(x):
        _check(_lib.ds_moe_route_dispatch(_ptr(router_logits), _ptr(x), T, H, E, top_k, _ptr(idx),
                                          _ptr(w), _ptr(off), _ptr(slot_of), _ptr(tmap), _ptr(disp),
                                          _ptr(ws), need, _stream(x)), "moe_route_dispatch")
    return idx, w, off, slot_of, tmap, disp


def moe_expert_mlp(rows: torch.Tensor, group_offsets: torch.Tensor, packed_w1: torch.Tensor,
                   w2: torch.Tensor, out: Optional[torch.Tensor] = None,
                   out_row_map: Optional[torch.Tensor] = None,
                   h: Optional[torch.Tensor] = None, max_ctas: int = 0) -> torch.Tensor:
    """Grouped SwiGLU expert MLP over expert-major rows (GEMM1+SwiGLU, GEMM2)."""
    R, H = rows.shape
    G, two_i, _ = packed_w1.shape
    I = two_i // 2
    if out is None:
        out = torch.empty((R, H), dtype=torch.bfloat16, device=rows.device)
    if h is None:
        h = torch.empty((R, I), dtype=torch.bfloat16, device=rows.device)
    if R == 0:
        return out
    with _on_device(rows):
        _check(_lib.ds_moe_expert_mlp(_ptr(rows), R, _ptr(group_offsets), G, _ptr(packed_w1),
                                      _ptr(w2), H, I, _ptr(h), _ptr(out), _ptr(out_row_map),
                                      int(max_ctas), _stream(rows)), "moe_expert_mlp")
    return out


def dense_mlp(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor,
              out: Optional[torch.Tensor] = None, max_ctas: int = 0) -> torch.Tensor:
    """One SwiGLU MLP over all rows (the shared expert): w1 [2I, H], w2 [H, I]."""
    R, H = x.shape
    I = w1.shape[0] // 2
    if out is None:
        out = torch.empty((R, H), dtype=torch.bfloat16, device=x.device)
    if R == 0:
        return out
    h = torch.empty((R, I), dtype=torch.bfloat16, device=x.device)
    with _on_device(x):
        _check(_lib.ds_dense_mlp(_ptr(x), R, _ptr(w1), _ptr(w2), H, I, _ptr(h), _ptr(out),
                                 int(max_ctas), _stream(x)), "dense_mlp")
    return out


def dense_mlp_ws(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor,
                 workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """dense_mlp whose GEMMs split K over the SMs when there are few rows (decode)."""
    R, H = x.shape
    I = w1.shape[0] // 2
    out = torch.empty((R, H), dtype=torch.bfloat16, device=x.device)
    if R == 0:
        return out
    h = torch.empty((R, I), dtype=torch.bfloat16, device=x.device)
    need = int(_lib.ds_dense_mlp_workspace_size(R, H, I))
    if workspace is None or workspace.numel() < need:
        workspace = _workspace(need, x.device)
    with _on_device(x):
        _check(_lib.ds_dense_mlp_ws(_ptr(x), R, _ptr(w1), _ptr(w2), H, I, _ptr(h), _ptr(out),
                                    _ptr(workspace), workspace.numel(), _stream(x)), "dense_mlp")
    return out


def moe_combine_slots(expert_out: torch.Tensor, slot_of: torch.Tensor, topk_weights: torch.Tensor,
                      shared_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out[t] = sum_j w[t,j] * expert_out[slot_of[t,j]] (+ shared_out[t]), one bf16 rounding."""
    T, k = slot_of.shape
    H = expert_out.shape[1]
    out = torch.empty((T, H), dtype=torch.bfloat16, device=expert_out.device)
    if T == 0:
        return out
    with _on_device(expert_out):
        _check(_lib.ds_moe_combine_slots(_ptr(expert_out), _ptr(slot_of), _ptr(topk_weights), k,
                                         _ptr(shared_out), _ptr(out), T, H, _stream(expert_out)),
               "moe_combine_slots")
    return out


def ep_plan(recv_counts: torch.Tensor, recv_rows: int):
    """Receive-side plan of the expert-parallel all-to-all: recv_counts int32 [N, El] ->
    (expert_offsets [El+1], row_map [recv_rows])."""
    N, El = recv_counts.shape
    dev = recv_counts.device
    off = torch.empty((El + 1,), dtype=torch.int32, device=dev)
    row_map = torch.empty((max(recv_rows, 1),), dtype=torch.int32, device=dev)
    need = _lib.ds_ep_plan_workspace_size(N, El)
    ws = _workspace(need, dev)
    with _on_device(recv_counts):
        _check(_lib.ds_ep_plan(_ptr(recv_counts.contiguous()), N, El, recv_rows, _ptr(off),
                               _ptr(row_map), _ptr(ws), need, _stream(recv_counts)), "ep_plan")
    return off, row_map[:recv_rows]


def gather_rows(src: torch.Tensor, row_map: torch.Tensor,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
    R = row_map.shape[0]
    H = src.shape[1]
    if out is None:
        out = torch.empty((R, H), dtype=src.dtype, device=src.device)
    if R == 0:
        return out
    with _on_device(src):
        _check(_lib.ds_gather_rows(_ptr(src), _ptr(row_map), R, H, _ptr(out), _stream(src)),
               "gather_rows")
    return out


def router_weight_split(gate_weight: torch.Tensor) -> torch.Tensor:
    """f32 gate [E, H] -> bf16 [256, H]: hi/mid/lo parts (rows e, 64+e, 128+e) summing to it."""
    g = gate_weight.detach().float().contiguous()
    E, H = g.shape
    out = torch.empty((256, H), dtype=torch.bfloat16, device=g.device)
    with _on_device(g):
        _check(_lib.ds_router_weight_split(_ptr(g), E, H, _ptr(out), _stream(g)),
               "router_weight_split")
    return out


def moe_router(x: torch.Tensor, w_split: torch.Tensor, num_experts: int, top_k: int = 6,
               logits_out: Optional[torch.Tensor] = None):
    """Router GEMM (f32-accurate, tensor cores) + top-k: -> (idx [T,k] i32, w [T,k] f32).
    `logits_out` (f32 [T, E]) optionally receives the summed logits."""
    _check_tensor(x, "x", torch.bfloat16, "bfloat16", 2, "[T, H]")
    T, H = x.shape
    idx = torch.empty((T, top_k), dtype=torch.int32, device=x.device)
    w = torch.empty((T, top_k), dtype=torch.float32, device=x.device)
    if T == 0:
        return idx, w
    need = _lib.ds_moe_router_workspace_size(T)
    ws = _workspace(need, x.device)
    with _on_device(x):
        _check(_lib.ds_moe_router(_ptr(x), _ptr(w_split), T, H, num_experts, top_k, _ptr(idx),
                                  _ptr(w), _ptr(logits_out), _ptr(ws), need, _stream(x)),
               "moe_router")
    return idx, w


def moe_dispatch_routed(idx: torch.Tensor, w: torch.Tensor, x: torch.Tensor, num_experts: int):
    """Offsets + deterministic dispatch from given routing -> (offsets, slot_of, token_map,
    dispatched)."""
    T, H = x.shape
    k = idx.shape[1]
    dev = x.device
    off = torch.empty((num_experts + 1,), dtype=torch.int32, device=dev)
    slot_of = torch.empty((T, k), dtype=torch.int32, device=dev)
    tmap = torch.empty((T * k,), dtype=torch.int32, device=dev)
    disp = torch.empty((T * k, H), dtype=torch.bfloat16, device=dev)
    need = _lib.ds_moe_route_dispatch_workspace_size(T, num_experts, k)
    ws = _workspace(need, dev)
    with _on_device(x):
        _check(_lib.ds_moe_dispatch_routed(_ptr(idx), _ptr(w), _ptr(x), T, H, num_experts, k,
                                           _ptr(off), _ptr(slot_of), _ptr(tmap), _ptr(disp),
                                           _ptr(ws), need, _stream(x)), "moe_dispatch_routed")
    return off, slot_of, tmap, disp


def _check_out(out: torch.Tensor, T: int, H: int, device) -> None:
    _require(out.dtype == torch.bfloat16 and tuple(out.shape) == (T, H) and out.is_contiguous()
             and out.device == device, "out must be a contiguous bf16 [T, H] tensor on x's device")


def moe_layer_forward_from_x(x: torch.Tensor, router_w_split: torch.Tensor, num_experts: int,
                             packed_w1: torch.Tensor, w2: torch.Tensor,
                             shared_w1: Optional[torch.Tensor] = None,
                             shared_w2: Optional[torch.Tensor] = None, top_k: int = 6,
                             out: Optional[torch.Tensor] = None,
                             workspace: Optional[torch.Tensor] = None,
                             events: Optional[Sequence[torch.cuda.Event]] = None,
                             logits_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Whole MoE layer from the tokens in one C call, router included (f32-accurate tensor-core
    router + top-k epilogue).  `logits_out` (f32 [T, E]) receives the router logits."""
    _check_tensor(x, "x", torch.bfloat16, "bfloat16", 2, "[T, H]")
    T, H = x.shape
    E = num_experts
    I = packed_w1.shape[1] // 2
    _require(packed_w1.shape[0] == E and tuple(w2.shape) == (E, H, I), "expert weight shapes")
    Is = 0 if shared_w1 is None else shared_w1.shape[0] // 2
    if out is None:
        out = torch.empty((T, H), dtype=torch.bfloat16, device=x.device)
    else:
        _check_out(out, T, H, x.device)
    if T == 0:
        return out
    need = moe_layer_workspace_size(T, H, E, top_k, I, Is)
    if workspace is None or workspace.numel() < need:
        workspace = _workspace(need, x.device)
    ev = None
    if events is not None:
        _require(len(events) == LAYER_NUM_EVENTS, f"events must hold {LAYER_NUM_EVENTS} events")
        st = torch.cuda.current_stream(x.device)
        for e in events:
            e.record(st)
        ev = (ctypes.c_void_p * LAYER_NUM_EVENTS)(*[e.cuda_event for e in events])
    with _on_device(x):
        _check(_lib.ds_moe_layer_forward_from_x(
            _ptr(x), _ptr(router_w_split), _ptr(logits_out), _ptr(packed_w1), _ptr(w2),
            _ptr(shared_w1), _ptr(shared_w2), _ptr(out), T, H, E, top_k, I, Is, _ptr(workspace),
            workspace.numel(), ev, _stream(x)), "moe_layer_forward_from_x")
    return out


def moe_layer_fused(hidden_states: torch.Tensor, gate_weight: torch.Tensor,
                    packed_w1: torch.Tensor, w2: torch.Tensor,
                    shared_w1: Optional[torch.Tensor] = None,
                    shared_w2: Optional[torch.Tensor] = None, top_k: int = 6) -> torch.Tensor:
    """The whole MoE layer in one call from the router's gate weight (any float dtype,
    [E, H]): the additive op of this surface for callers that hold the gate as a tensor.  It
    splits the gate for the tensor-core router on every call; callers that run the layer
    repeatedly keep the split (`router_weight_split`) and call `moe_layer_forward_from_x`,
    as `moe_fused.FusedMoELayer` does."""
    split = router_weight_split(gate_weight.float().contiguous())
    return moe_layer_forward_from_x(hidden_states, split, gate_weight.shape[0], packed_w1, w2,
                                    shared_w1, shared_w2, top_k=top_k)


def dense_gemm1_swiglu(x: torch.Tensor, w1: torch.Tensor, max_ctas: int = 0) -> torch.Tensor:
    """h = silu(x @ gate^T) * (x @ up^T) with w1 = [gate; up] [2I, H] -> bf16 [R, I]."""
    R, H = x.shape
    I = w1.shape[0] // 2
    h = torch.empty((R, I), dtype=torch.bfloat16, device=x.device)
    if R == 0:
        return h
    with _on_device(x):
        _check(_lib.ds_dense_gemm1_swiglu(_ptr(x), R, _ptr(w1), H, I, _ptr(h), int(max_ctas),
                                          _stream(x)), "dense_gemm1_swiglu")
    return h


def dense_gemm2(h: torch.Tensor, w2: torch.Tensor, max_ctas: int = 0) -> torch.Tensor:
    """out = h @ w2^T, w2 [H, I] -> bf16 [R, H]."""
    R, I = h.shape
    H = w2.shape[0]
    out = torch.empty((R, H), dtype=torch.bfloat16, device=h.device)
    if R == 0:
        return out
    with _on_device(h):
        _check(_lib.ds_dense_gemm2(_ptr(h), R, _ptr(w2), I, H, _ptr(out), int(max_ctas),
                                   _stream(h)), "dense_gemm2")
    return out


# ---- expert parallelism over NVLink peer memory (symmetric segments via CUDA IPC) ---------

def ep_symmetric_size(max_tokens: int, hidden_size: int, num_experts: int, top_k: int,
                      world: int) -> int:
    n = _sz(0)
    _check(_lib.ds_ep_symmetric_size(max_tokens, hidden_size, num_experts, top_k, world,
                                     ctypes.byref(n)), "ep_symmetric_size")
    return n.value


def ep_alloc(nbytes: int, device: torch.device) -> int:
    """cudaMalloc'd, zero-filled segment on `device` (a raw pointer; free with ep_free)."""
    p = _vp()
    with torch.cuda.device(device):
        _check(_lib.ds_ep_alloc(nbytes, ctypes.byref(p)), "ep_alloc")
    return p.value


def ep_free(ptr: int, device: torch.device) -> None:
    with torch.cuda.device(device):
        _check(_lib.ds_ep_free(ptr), "ep_free")


def ep_ipc_handle(ptr: int, device: torch.device) -> bytes:
    buf = ctypes.create_string_buffer(EP_IPC_HANDLE_BYTES)
    with torch.cuda.device(device):
        _check(_lib.ds_ep_ipc_handle(ptr, buf), "ep_ipc_handle")
    return buf.raw


def ep_ipc_open(handle: bytes, device: torch.device) -> int:
    _require(len(handle) == EP_IPC_HANDLE_BYTES, "ep_ipc_open: bad handle size")
    p = _vp()
    buf = ctypes.create_string_buffer(bytes(handle), EP_IPC_HANDLE_BYTES)
    with torch.cuda.device(device):
        _check(_lib.ds_ep_ipc_open(buf, ctypes.byref(p)), "ep_ipc_open")
    return p.value


def ep_ipc_close(ptr: int, device: torch.device) -> None:
    with torch.cuda.device(device):
        _check(_lib.ds_ep_ipc_close(ptr), "ep_ipc_close")


def ep_layer_workspace_size(max_tokens: int, hidden_size: int, num_experts: int, top_k: int,
                            intermediate_size: int, shared_intermediate_size: int,
                            world: int) -> int:
    return int(_lib.ds_ep_layer_workspace_size(max_tokens, hidden_size, num_experts, top_k,
                                               intermediate_size, shared_intermediate_size,
                                               world))


def ep_layer_forward(x: torch.Tensor, router_w_split: torch.Tensor, num_experts: int,
                     w1_local: torch.Tensor, w2_local: torch.Tensor,
                     shared_w1: Optional[torch.Tensor], shared_w2: Optional[torch.Tensor],
                     top_k: int, rank: int, world: int, max_tokens: int,
                     sym_bases: Sequence[int], epoch: int, workspace: torch.Tensor,
                     out: Optional[torch.Tensor] = None, timeout_ms: int = 10000,
                     events: Optional[Sequence[torch.cuda.Event]] = None,
                     logits_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One expert-parallel MoE layer forward of this rank's tokens (every rank calls it for
    every forward with the same epoch sequence 1, 2, ...).  w1_local [El, 2I, H] and
    w2_local [El, H, I] hold this rank's experts; sym_bases[r] = rank r's symmetric segment
    as mapped in this process."""
    _check_tensor(x, "x", torch.bfloat16, "bfloat16", 2, "[T, H]")
    T, H = x.shape
    E = num_experts
    El = w1_local.shape[0]
    I = w1_local.shape[1] // 2
    _require(El * world == E and tuple(w2_local.shape) == (El, H, I), "local expert weight shapes")
    Is = 0 if shared_w1 is None else shared_w1.shape[0] // 2
    if out is None:
        out = torch.empty((T, H), dtype=torch.bfloat16, device=x.device)
    else:
        _check_out(out, T, H, x.device)
    need = ep_layer_workspace_size(max_tokens, H, E, top_k, I, Is, world)
    _require(workspace.numel() >= need, f"ep_layer_forward: workspace needs {need} bytes")
    ev = None
    if events is not None:
        _require(len(events) == EP_NUM_EVENTS, f"events must hold {EP_NUM_EVENTS} events")
        st = torch.cuda.current_stream(x.device)
        for e in events:
            e.record(st)
        ev = (ctypes.c_void_p * EP_NUM_EVENTS)(*[e.cuda_event for e in events])
    bases = (ctypes.c_void_p * world)(*sym_bases)
    with _on_device(x):
        _check(_lib.ds_ep_layer_forward(
            _ptr(x) if T else None, T, _ptr(router_w_split), _ptr(logits_out), _ptr(w1_local),
            _ptr(w2_local), _ptr(shared_w1), _ptr(shared_w2), _ptr(out) if T else None, H, E,
            top_k, I, Is, rank, world, max_tokens, bases, epoch, timeout_ms, _ptr(workspace),
            workspace.numel(), ev, _stream(x)), "ep_layer_forward")
    return out


# ---- torch custom operators ----------------------------------------------------------------
# Every drop-in op is also registered as torch.ops.ds_kernels.<name> (torch_ops.py) with a
# fake kernel, so torch.compile / torch.export / FakeTensor propagation see through it.  The
# module-level functions stay direct C-ABI calls in eager mode and route through the
# registered operator while torch.compile traces them.
import functools as _functools  # noqa: E402

_eager = {}


def _traced(name):
    eager = globals()[name]
    _eager[name] = eager

    @_functools.wraps(eager)
    def op(*args, **kwargs):
        if torch.compiler.is_compiling():
            r = getattr(torch.ops.ds_kernels, name)(*args, **kwargs)
            return list(r) if isinstance(r, tuple) else r
        return eager(*args, **kwargs)

    return op


_TRACED_OPS = ("moe_routing", "moe_scan", "moe_dispatch", "moe_combine", "swiglu", "moe_gemm1",
               "moe_gemm2", "rms_norm", "kv_upproj", "rope", "moe_gemm1_swiglu",
               "rms_norm_residual", "moe_layer_fused")
for _n in _TRACED_OPS:
    globals()[_n] = _traced(_n)
del _n

from . import torch_ops  # noqa: E402,F401  (registers torch.ops.ds_kernels.*)
