"""CPU restatement of the reference MLA projection ops (test infrastructure only).

rms_norm   : src/reference/mla.py:59-64 (f32 statistics), one rounding at the end as in
             src/kernels/mla/rms_norm.cu:104-114.
rms_norm_residual: the residual add + pre-norm of src/reference/decoder_layer.py:123-139.
yarn_cos_sin: the YaRN tables of src/reference/mla.py:66-173 (correction range, linear ramp,
             frequency blend, mscale ratio), restated.
rope       : src/reference/mla.py:176-206 (interleave -> half transform, then
             q*cos + rotate_half(q)*sin).
kv_upproj  : F.linear(normed, W) in f32 (src/kernels/mla/kv_upproj.cu:77-119).
mla_attention: the causal scaled-dot-product step of src/reference/mla.py:355-378.
mla_forward: the whole DeepSeekMLA.forward of src/reference/mla.py:295-393 in f32 (q_proj,
             kv_a_proj_with_mqa, kv_a_layernorm, kv_b_proj, RoPE on the 64-wide parts,
             causal attention over 192-wide q/k and 128-wide v, o_proj).
mla_decode_step: the same forward for one new token per sequence whose predecessors are
             given as the raw latents / raw k_pe of a latent KV cache (src/kernels/
             mla_cache.py:29-219 stores exactly those): the last row of mla_forward when the
             cache holds the prefix's projections.
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


def mla_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                  softmax_scale: float) -> torch.Tensor:
    """q, k [b, h, s, dqk], v [b, h, s, dv] -> [b, h, s, dv] in f32: causal softmax(q k^T *
    scale) v with the upper triangle masked to -inf (src/reference/mla.py:355-378)."""
    qf, kf, vf = q.to(F32), k.to(F32), v.to(F32)
    s_len = qf.shape[2]
    w = torch.matmul(qf, kf.transpose(2, 3)) * softmax_scale
    mask = torch.triu(torch.full((s_len, s_len), float("-inf")), diagonal=1)
    w = torch.softmax(w + mask, dim=-1)
    return torch.matmul(w, vf)


def mla_forward(x: torch.Tensor, w_q: torch.Tensor, w_kva: torch.Tensor, norm_w: torch.Tensor,
                w_kvb: torch.Tensor, w_o: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                softmax_scale: float, heads: int, eps: float = 1e-6,
                return_aux: bool = False):
    """DeepSeekMLA.forward (src/reference/mla.py:295-393) in f32 with positions 0..s-1.

    x [b, s, hidden]; w_q [heads*192, hidden]; w_kva [512+64, hidden]; norm_w [512];
    w_kvb [heads*(128+128), 512]; w_o [hidden, heads*128]; cos/sin [>= s, 64]."""
    b, s_len, _ = x.shape
    xf = x.to(F32)
    q = (xf @ w_q.to(F32).t()).view(b, s_len, heads, 192).transpose(1, 2)
    q_nope, q_pe = q[..., :128], q[..., 128:]
    ckv = xf @ w_kva.to(F32).t()
    latent, k_pe = ckv[..., :512], ckv[..., 512:]
    k_pe = k_pe.view(b, s_len, 1, 64).transpose(1, 2)
    kv = (rms_norm(latent, norm_w, eps) @ w_kvb.to(F32).t()).view(b, s_len, heads, 256)
    kv = kv.transpose(1, 2)
    k_nope, v = kv[..., :128], kv[..., 128:]
    c = cos[:s_len].to(F32)[None, None]
    sn = sin[:s_len].to(F32)[None, None]
    q_pe, k_pe = rope(q_pe, k_pe, c, sn)
    qs = torch.cat([q_nope, q_pe], dim=-1)
    ks = torch.cat([k_nope, k_pe.expand(b, heads, s_len, 64)], dim=-1)
    o = mla_attention(qs, ks, v, softmax_scale)
    attn = o.transpose(1, 2).reshape(b, s_len, heads * 128)
    out = attn @ w_o.to(F32).t()
    if return_aux:
        return out, {"query_states": qs, "key_states": ks, "value": v, "attn": attn}
    return out


def mla_forward_rows(x: torch.Tensor, w_q: torch.Tensor, w_kva: torch.Tensor,
                     norm_w: torch.Tensor, w_kvb: torch.Tensor, w_o: torch.Tensor,
                     cos: torch.Tensor, sin: torch.Tensor, softmax_scale: float, heads: int,
                     rows: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """mla_forward restricted to the output rows `rows` (token indices, the same for every
    sequence): keys and values of every token, queries and attention only for those rows, so
    full-length sequences stay cheap to check.  Returns f32 [b, len(rows), hidden]."""
    b, s_len, _ = x.shape
    xf = x.to(F32)
    rows = rows.to(torch.long)
    R = rows.numel()
    q = (xf[:, rows] @ w_q.to(F32).t()).view(b, R, heads, 192).transpose(1, 2)
    q_nope, q_pe = q[..., :128], q[..., 128:]
    ckv = xf @ w_kva.to(F32).t()
    latent, k_pe = ckv[..., :512], ckv[..., 512:]
    k_pe = k_pe.view(b, s_len, 1, 64).transpose(1, 2)
    kv = (rms_norm(latent, norm_w, eps) @ w_kvb.to(F32).t()).view(b, s_len, heads, 256)
    kv = kv.transpose(1, 2)
    k_nope, v = kv[..., :128], kv[..., 128:]
    _, k_pe = rope(k_pe, k_pe, cos[:s_len].to(F32)[None, None], sin[:s_len].to(F32)[None, None])
    q_pe, _ = rope(q_pe, q_pe[:, :1], cos[rows].to(F32)[None, None], sin[rows].to(F32)[None, None])
    qs = torch.cat([q_nope, q_pe], dim=-1)
    ks = torch.cat([k_nope, k_pe.expand(b, heads, s_len, 64)], dim=-1)
    w = torch.matmul(qs, ks.transpose(2, 3)) * softmax_scale
    masked = torch.arange(s_len)[None, :] > rows[:, None]
    w = torch.softmax(w.masked_fill(masked[None, None], float("-inf")), dim=-1)
    attn = torch.matmul(w, v).transpose(1, 2).reshape(b, R, heads * 128)
    return attn @ w_o.to(F32).t()


def mla_decode_step(x_new: torch.Tensor, cache_latent: torch.Tensor, cache_kpe: torch.Tensor,
                    w_q: torch.Tensor, w_kva: torch.Tensor, norm_w: torch.Tensor,
                    w_kvb: torch.Tensor, w_o: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                    softmax_scale: float, heads: int, eps: float = 1e-6) -> torch.Tensor:
    """x_new [b, hidden] at position L = cache_latent.shape[1]; cache_latent [b, L, 512] and
    cache_kpe [b, L, 64] the raw latents / k_pe of positions 0 .. L-1.  Returns f32
    [b, hidden]: DeepSeekMLA.forward's output row L (src/reference/mla.py:295-393)."""
    b, L, _ = cache_latent.shape
    xf = x_new.to(F32)
    q = (xf @ w_q.to(F32).t()).view(b, heads, 1, 192)
    ckv = xf @ w_kva.to(F32).t()
    latent = torch.cat([cache_latent.to(F32), ckv[:, None, :512]], dim=1)    # [b, L+1, 512]
    kpe = torch.cat([cache_kpe.to(F32), ckv[:, None, 512:]], dim=1)          # [b, L+1, 64]
    kv = (rms_norm(latent, norm_w, eps) @ w_kvb.to(F32).t()).view(b, L + 1, heads, 256)
    kv = kv.transpose(1, 2)
    k_nope, v = kv[..., :128], kv[..., 128:]
    _, k_rot = rope(kpe[:, None], kpe[:, None], cos[:L + 1].to(F32)[None, None],
                    sin[:L + 1].to(F32)[None, None])
    q_rot, _ = rope(q[..., 128:], q[..., 128:][:, :1], cos[L:L + 1].to(F32)[None, None],
                    sin[L:L + 1].to(F32)[None, None])
    qs = torch.cat([q[..., :128], q_rot], dim=-1)                             # [b, h, 1, 192]
    ks = torch.cat([k_nope, k_rot.expand(b, heads, L + 1, 64)], dim=-1)       # [b, h, L+1, 192]
    w = torch.softmax(torch.matmul(qs, ks.transpose(2, 3)) * softmax_scale, dim=-1)
    attn = torch.matmul(w, v).reshape(b, heads * 128)
    return attn @ w_o.to(F32).t()
