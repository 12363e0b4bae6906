"""Fused MLA (multi-head latent attention) forward: drop-in for the reference's DeepSeekMLA.

    FusedMLA(mla_module)(hidden_states)      (src/reference/mla.py:209-393)

Reads the module's weights once (q_proj, kv_a_proj_with_mqa, kv_a_layernorm, kv_b_proj,
o_proj), its RoPE tables (rotary_emb.cos_cached / sin_cached: YaRN or plain) and its
softmax_scale, and runs every forward as ONE C call (ds_mla_forward): the q and kv_a
projections as one tcgen05 GEMM, the latent RMSNorm, the kv_b projection, RoPE in place on
the 64-wide parts, the causal attention kernel (S = Q K^T and O += P V on the tensor cores,
online softmax in between) and o_proj, on the current stream with no host synchronisation.

Causal attention only (the reference builds the causal mask itself when attention_mask is
None, mla.py:362-369); an explicit attention_mask is refused.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

import ds_kernels


class FusedMLA(nn.Module):
    """Runs DeepSeekMLA's forward on the sm_100a kernels; outputs bf16."""

    def __init__(self, mla_module: nn.Module, device: Optional[torch.device] = None):
        super().__init__()
        m = mla_module
        dev = device if device is not None else m.q_proj.weight.device
        if dev.type != "cuda":
            raise RuntimeError("FusedMLA: the module (or `device`) must be on a CUDA device")
        self.heads = m.num_heads
        self.hidden = m.hidden_size
        if (m.qk_nope_head_dim, m.qk_rope_head_dim, m.v_head_dim, m.kv_lora_rank) != (128, 64, 128, 512):
            raise ValueError("FusedMLA: head sizes must be 128 nope + 64 rope, v 128, latent 512")
        bf = torch.bfloat16
        self.w_qkv_a = torch.cat([m.q_proj.weight.detach(),
                                  m.kv_a_proj_with_mqa.weight.detach()]).to(dev, bf).contiguous()
        self.kv_norm_weight = m.kv_a_layernorm.weight.detach().to(dev, torch.float32).contiguous()
        self.eps = float(m.kv_a_layernorm.variance_epsilon)
        self.w_kv_b = m.kv_b_proj.weight.detach().to(dev, bf).contiguous()
        self.w_o = m.o_proj.weight.detach().to(dev, bf).contiguous()
        self.cos = m.rotary_emb.cos_cached.detach().to(dev, bf).contiguous()
        self.sin = m.rotary_emb.sin_cached.detach().to(dev, bf).contiguous()
        self.softmax_scale = float(m.softmax_scale)
        self._ws: Optional[torch.Tensor] = None

    def forward(self, hidden_states: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
                position_ids: Optional[torch.Tensor] = None, events=None) -> torch.Tensor:
        if attention_mask is not None:
            raise NotImplementedError("FusedMLA: causal attention only (attention_mask=None)")
        x = hidden_states.to(torch.bfloat16)
        B, S, _ = x.shape
        need = ds_kernels.mla_forward_workspace_size(B, S, self.hidden, self.heads)
        if self._ws is None or self._ws.numel() < need or self._ws.device != x.device:
            self._ws = torch.empty(max(need, 1), dtype=torch.uint8, device=x.device)
        return ds_kernels.mla_forward(x, self.w_qkv_a, self.kv_norm_weight, self.w_kv_b,
                                      self.w_o, self.cos, self.sin, self.softmax_scale,
                                      self.heads, position_ids=position_ids, eps=self.eps,
                                      workspace=self._ws, events=events)
