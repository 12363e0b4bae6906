"""CPU restatement of the reference MLA projection ops (test infrastructure only).

rms_norm   : src/reference/mla.py:59-64 (f32 statistics), one rounding at the end as in
             src/kernels/mla/rms_norm.cu:104-114.
rms_norm_residual: the residual add + pre-norm of src/reference/decoder_layer.py:123-139.
yarn_cos_sin: the YaRN tables of src/reference/mla.py:66-173 (correction range, linear ramp,
             frequency blend, mscale ratio), restated.
rope       : src/reference/mla.py:176-206 (interleave -> half transform, then
             q*cos + rotate_half(q)*sin).
kv_upproj  : F.linear(normed, W) in f32 (src/kernels/mla/kv_upproj.cu:77-119).
"""
from __future__ import annotations

import math
from typing import Tuple

import torch

F32 = torch.float32


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    xf = x.to(F32)
    var = xf.pow(2).mean(-1, keepdim=True)
    return weight.to(F32) * (xf * torch.rsqrt(var + eps))


def rms_norm_residual(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                      eps: float = 1e-6) -> Tuple[torch.Tensor, torch.Tensor]:
    """(normed, sum): sum = residual + x as bf16 tensors add (src/reference/decoder_layer.py:
    130, 133-135), normed = rms_norm(sum) (src/reference/mla.py:59-64)."""
    s = (residual.to(F32) + x.to(F32)).to(torch.bfloat16)
    return rms_norm(s, weight, eps), s


def _correction_dim(num_rot: float, dim: int, base: float, max_pos: int) -> float:
    return (dim * math.log(max_pos / (num_rot * 2 * math.pi))) / (2 * math.log(base))


def _mscale(scale: float, m: float) -> float:
    return 1.0 if scale <= 1 else 0.1 * m * math.log(scale) + 1.0


def yarn_cos_sin(seq_len: int, dim: int = 64, base: float = 10000.0, scaling_factor: float = 40.0,
                 original_max_position_embeddings: int = 4096, beta_fast: float = 32,
                 beta_slow: float = 1, mscale: float = 0.707,
                 mscale_all_dim: float = 0.707) -> Tuple[torch.Tensor, torch.Tensor]:
    """cos/sin tables [seq_len, dim] (f32).  scaling_factor=1 gives plain RoPE with theta=base."""
    pos_freq = base ** (torch.arange(0, dim, 2, dtype=F32) / dim)
    f_extra = 1.0 / pos_freq
    f_inter = 1.0 / (scaling_factor * pos_freq)
    lo = max(math.floor(_correction_dim(beta_fast, dim, base, original_max_position_embeddings)), 0)
    hi = min(math.ceil(_correction_dim(beta_slow, dim, base, original_max_position_embeddings)),
             dim - 1)
    if lo == hi:
        hi += 0.001
    ramp = torch.clamp((torch.arange(dim // 2, dtype=F32) - lo) / (hi - lo), 0, 1)
    extra_mask = 1.0 - ramp
    inv_freq = f_inter * (1 - extra_mask) + f_extra * extra_mask
    t = torch.arange(seq_len, dtype=F32)
    freqs = torch.outer(t, inv_freq)
    emb = torch.cat((freqs, freqs), dim=-1)
    m = float(_mscale(scaling_factor, mscale) / _mscale(scaling_factor, mscale_all_dim))
    return emb.cos() * m, emb.sin() * m


def rope(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor,
         sin: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """q [b, h, s, d], k [b, 1, s, d]; cos/sin broadcastable to [b, 1, s, d] (pre-indexed)."""
    def one(x):
        b, h, s, d = x.shape
        xd = x.to(F32).view(b, h, s, d // 2, 2).transpose(4, 3).reshape(b, h, s, d)
        half = d // 2
        rot = torch.cat((-xd[..., half:], xd[..., :half]), dim=-1)
        return xd * cos.to(F32) + rot * sin.to(F32)
    return one(q), one(k)


def kv_upproj(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    return x.to(F32) @ w.to(F32).t()
