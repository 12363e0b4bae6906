"""Latent KV cache for MLA decode: drop-in for src/kernels/mla_cache.py:29-219.

Same constructor, properties (`current_len`, `remaining_capacity`, `memory_bytes`), methods
(`update`, `get`, `reset`, `for_inference`) and error messages as the reference's
LatentKVCache: per sequence and position it stores the raw, pre-norm 512-wide latent
(`kv_latent`) and the raw, un-rotated 64-wide k_pe (`k_pe_cache`), pre-allocated to
`max_seq`, written at the current length and read back as zero-copy views.

On a CUDA device it also keeps two side arrays for the decode kernel
(ds_kernels.mla_decode_step): `rstd` (f32 [bsz, max_seq]: the latent RMSNorm's row scale
rsqrt(mean(latent^2) + eps)) and `k_pe_rot` (bf16 [bsz, max_seq, 64]: k_pe rotated at its
position).  The fused paths (FusedMLA.prefill / FusedMLA.decode) write them together with the
raw values; positions written through the reference's `update()` (which has no RoPE tables)
get them on the next decode step.  `memory_bytes` counts the two reference buffers, as the
reference does; `side_bytes` the side arrays.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch


class LatentKVCache:
    def __init__(self, bsz: int, max_seq: int, kv_lora_rank: int = 512, rope_head_dim: int = 64,
                 device: str = "cuda", dtype: torch.dtype = torch.bfloat16):
        if not isinstance(bsz, int) or bsz < 1:
            raise ValueError(f"bsz must be a positive integer, got {bsz}")
        if not isinstance(max_seq, int) or max_seq < 1:
            raise ValueError(f"max_seq must be a positive integer, got {max_seq}")
        self.bsz = bsz
        self.max_seq = max_seq
        self.kv_lora_rank = kv_lora_rank
        self.rope_head_dim = rope_head_dim
        self.device = torch.device(device)
        self.dtype = dtype
        self._len = 0
        self.kv_latent = torch.zeros((bsz, max_seq, kv_lora_rank), dtype=dtype, device=self.device)
        self.k_pe_cache = torch.zeros((bsz, max_seq, rope_head_dim), dtype=dtype, device=self.device)
        # side arrays of the decode kernel (CUDA only); valid for positions < _side_len
        self._side_len = 0
        if self.device.type == "cuda":
            self.rstd = torch.zeros((bsz, max_seq), dtype=torch.float32, device=self.device)
            self.k_pe_rot = torch.zeros((bsz, max_seq, rope_head_dim), dtype=dtype,
                                        device=self.device)
            # the length on the device: the decode kernels read the position from it and
            # advance it, so a captured CUDA graph of a decode step replays at successive
            # positions (the host-side length is advanced alongside)
            self.len_dev = torch.zeros((1,), dtype=torch.int32, device=self.device)
        else:
            self.rstd = self.k_pe_rot = self.len_dev = None

    # ---- properties (reference surface) --------------------------------------------------
    @property
    def current_len(self) -> int:
        """Number of tokens currently stored in the cache."""
        return self._len

    @property
    def remaining_capacity(self) -> int:
        """Number of additional tokens that can be appended."""
        return self.max_seq - self._len

    @property
    def memory_bytes(self) -> int:
        """Total bytes consumed by both cache buffers."""
        return (self.kv_latent.numel() + self.k_pe_cache.numel()) * self.kv_latent.element_size()

    @property
    def side_bytes(self) -> int:
        """Bytes of the decode kernel's side arrays (0 off CUDA)."""
        if self.rstd is None:
            return 0
        return self.rstd.numel() * 4 + self.k_pe_rot.numel() * self.k_pe_rot.element_size()

    # ---- core operations (reference surface) ---------------------------------------------
    def update(self, compressed_kv: torch.Tensor, k_pe: torch.Tensor) -> None:
        """Append new tokens: compressed_kv [bsz, new_tokens, kv_lora_rank], k_pe
        [bsz, new_tokens, rope_head_dim] (the raw k_pe, without the head dim)."""
        if compressed_kv.dim() != 3:
            raise ValueError(
                f"compressed_kv must be 3D [bsz, new_tokens, kv_lora_rank], "
                f"got shape {tuple(compressed_kv.shape)}")
        if k_pe.dim() != 3:
            raise ValueError(
                f"k_pe must be 3D [bsz, new_tokens, rope_head_dim], got shape {tuple(k_pe.shape)}")
        new_tokens = compressed_kv.shape[1]
        if self._len + new_tokens > self.max_seq:
            raise RuntimeError(
                f"KV cache overflow: current_len={self._len}, new_tokens={new_tokens}, "
                f"max_seq={self.max_seq}. Increase max_seq or reset the cache.")
        slot = slice(self._len, self._len + new_tokens)
        self.kv_latent[:, slot, :] = compressed_kv.to(self.device, self.dtype)
        self.k_pe_cache[:, slot, :] = k_pe.to(self.device, self.dtype)
        self._len += new_tokens
        if self.len_dev is not None:
            self.len_dev.fill_(self._len)

    def get(self, seq_len: Optional[int] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """(kv_latent [bsz, seq_len, kv_lora_rank], k_pe [bsz, seq_len, rope_head_dim]) views."""
        if seq_len is None:
            seq_len = self._len
        if seq_len > self._len:
            raise ValueError(f"Requested seq_len={seq_len} but cache only has {self._len} tokens.")
        return self.kv_latent[:, :seq_len, :], self.k_pe_cache[:, :seq_len, :]

    def reset(self) -> None:
        """Clear the cache for a new sequence (keeps the memory)."""
        self._len = 0
        self._side_len = 0
        if self.len_dev is not None:
            self.len_dev.zero_()

    def __repr__(self) -> str:
        used_mb = (self._len * (self.kv_lora_rank + self.rope_head_dim)
                   * self.kv_latent.element_size() * self.bsz) / (1024 ** 2)
        total_mb = self.memory_bytes / (1024 ** 2)
        return (f"LatentKVCache(bsz={self.bsz}, tokens={self._len}/{self.max_seq}, "
                f"used={used_mb:.2f}MB/{total_mb:.2f}MB, device={self.device}, dtype={self.dtype})")

    @classmethod
    def for_inference(cls, bsz: int, max_seq: int = 4096, device: str = "cuda") -> "LatentKVCache":
        """BF16 cache with the production defaults (512-wide latent, 64-wide k_pe)."""
        return cls(bsz=bsz, max_seq=max_seq, kv_lora_rank=512, rope_head_dim=64, device=device,
                   dtype=torch.bfloat16)

    # ---- decode-kernel bookkeeping ----------------------------------------------------------
    def _require_decode_layout(self) -> None:
        if self.rstd is None or self.dtype != torch.bfloat16 or self.kv_lora_rank != 512 \
                or self.rope_head_dim != 64:
            raise RuntimeError("the fused MLA kernels need a bf16 CUDA cache with a 512-wide "
                               "latent and a 64-wide k_pe")

    def _sync_side(self, cos: torch.Tensor, sin: torch.Tensor, eps: float) -> None:
        """Fill the side arrays of positions written through update() (raw values only)."""
        self._require_decode_layout()
        if self._side_len < self._len:
            import ds_kernels
            s0, s1 = self._side_len, self._len
            ds_kernels.mla_cache_append(self.kv_latent[:, s0:s1], self.k_pe_cache[:, s0:s1], self,
                                        s0, cos, sin, eps, copy_raw=False)
            self._side_len = s1

    def _advance(self, n: int, device_counted: bool) -> None:
        """A fused kernel appended n tokens, side arrays included (the callers bring the side
        arrays of earlier positions up to date before they launch); device_counted: the
        kernels already advanced len_dev."""
        if self._side_len < self._len:
            raise RuntimeError("LatentKVCache: side arrays were stale when tokens were appended")
        self._len += n
        self._side_len = self._len
        if not device_counted:
            self.len_dev.fill_(self._len)
