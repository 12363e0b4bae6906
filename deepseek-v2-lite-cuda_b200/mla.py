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

Decode (config 4) over a latent KV cache (mla_cache.LatentKVCache, the drop-in for
src/kernels/mla_cache.py): `prefill(prompt, cache)` runs the forward above and writes the
prompt's raw latents and k_pe into the cache; `decode(x, cache)` runs one token per sequence
through ds_mla_decode_step.  The decode weights absorb the kv_b projection (folded once, in
f32, rounded to bf16): the query weights become diag(g) W_uk_h^T W_q_nope_h per head (g the
latent norm weight) and the output weights W_o_h W_uv_h diag(g), so the attention scores and
values are taken against the 512-wide cached latent directly.
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
        self._dec_w = None
        self._dec_ws: Optional[torch.Tensor] = None

    @classmethod
    def from_weights(cls, w_q: torch.Tensor, w_kva: torch.Tensor, kv_norm_weight: torch.Tensor,
                     w_kvb: torch.Tensor, w_o: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                     softmax_scale: float, heads: int = 16, eps: float = 1e-6) -> "FusedMLA":
        """Build from the raw weights (the tensors DeepSeekMLA holds: q_proj [heads*192, H],
        kv_a_proj_with_mqa [576, H], kv_a_layernorm [512], kv_b_proj [heads*256, 512], o_proj
        [H, heads*128]) and the RoPE tables [positions, 64], all on one CUDA device."""
        self = cls.__new__(cls)
        nn.Module.__init__(self)
        bf = torch.bfloat16
        self.heads = heads
        self.hidden = w_q.shape[1]
        self.w_qkv_a = torch.cat([w_q.detach(), w_kva.detach()]).to(bf).contiguous()
        self.kv_norm_weight = kv_norm_weight.detach().float().contiguous()
        self.eps = float(eps)
        self.w_kv_b = w_kvb.detach().to(bf).contiguous()
        self.w_o = w_o.detach().to(bf).contiguous()
        self.cos = cos.detach().to(bf).contiguous()
        self.sin = sin.detach().to(bf).contiguous()
        self.softmax_scale = float(softmax_scale)
        self._ws = None
        self._dec_w = None
        self._dec_ws = None
        return self

    def decode_weights(self):
        """(w_dec bf16 [heads*(512+64) + 576, hidden], w_out bf16 [hidden, heads*512]): the
        absorbed decode weights, built once from the module's bf16 weights in f32."""
        if self._dec_w is None:
            H, hd = self.heads, self.hidden
            wq = self.w_qkv_a[:H * 192].float().view(H, 192, hd)
            wkva = self.w_qkv_a[H * 192:].float()
            wkvb = self.w_kv_b.float().view(H, 256, 512)
            g = self.kv_norm_weight.float()
            w_uk, w_uv = wkvb[:, :128], wkvb[:, 128:]                   # [H, 128, 512]
            w_qabs = torch.bmm(w_uk.transpose(1, 2), wq[:, :128]) * g[None, :, None]  # [H, 512, hd]
            w_dec = torch.cat([w_qabs.reshape(H * 512, hd), wq[:, 128:].reshape(H * 64, hd), wkva])
            wo = self.w_o.float().view(hd, H, 128).transpose(0, 1)        # [H, hd, 128]
            w_out = torch.bmm(wo, w_uv) * g[None, None, :]                # [H, hd, 512]
            w_out = w_out.transpose(0, 1).reshape(hd, H * 512)
            self._dec_w = (w_dec.to(torch.bfloat16).contiguous(),
                           w_out.to(torch.bfloat16).contiguous())
        return self._dec_w

    def prefill(self, hidden_states: torch.Tensor, cache) -> torch.Tensor:
        """forward() over a prompt at positions 0 .. seq-1 that also fills the (empty) cache."""
        x = hidden_states.to(torch.bfloat16)
        B, S, _ = x.shape
        need = ds_kernels.mla_forward_workspace_size(B, S, self.hidden, self.heads)
        if self._ws is None or self._ws.numel() < need or self._ws.device != x.device:
            self._ws = torch.empty(max(need, 1), dtype=torch.uint8, device=x.device)
        return ds_kernels.mla_prefill(x, self.w_qkv_a, self.kv_norm_weight, self.w_kv_b,
                                      self.w_o, self.cos, self.sin, self.softmax_scale,
                                      self.heads, cache, eps=self.eps, workspace=self._ws)

    def decode(self, hidden_states: torch.Tensor, cache, events=None) -> torch.Tensor:
        """One new token per sequence: hidden_states [bsz, hidden] or [bsz, 1, hidden] ->
        same shape; the token is appended to `cache` at its current length."""
        x = hidden_states.to(torch.bfloat16)
        x2 = x.reshape(x.shape[0], self.hidden).contiguous()
        if cache.current_len >= self.cos.shape[0]:
            raise RuntimeError("FusedMLA.decode: position beyond the RoPE tables")
        w_dec, w_out = self.decode_weights()
        need = ds_kernels.mla_decode_workspace_size(x2.shape[0], cache.max_seq, self.hidden)
        if self._dec_ws is None or self._dec_ws.numel() < need or self._dec_ws.device != x.device:
            self._dec_ws = torch.empty(max(need, 1), dtype=torch.uint8, device=x.device)
        out = ds_kernels.mla_decode_step(x2, w_dec, w_out, self.cos, self.sin, cache,
                                         self.softmax_scale, heads=self.heads, eps=self.eps,
                                         workspace=self._dec_ws, events=events)
        return out.view(x.shape)

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
