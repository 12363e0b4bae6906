"""LatentKVCache (mla_cache.py): the reference's cache surface (src/kernels/mla_cache.py:29-219)
on the CPU — constructor checks and messages, update / get / reset semantics, overflow, memory
accounting, for_inference.  The decode kernels' side arrays exist only on CUDA devices."""
import pytest
import torch

from mla_cache import LatentKVCache


def test_constructor_checks():
    with pytest.raises(ValueError, match="bsz must be a positive integer"):
        LatentKVCache(0, 8, device="cpu")
    with pytest.raises(ValueError, match="max_seq must be a positive integer"):
        LatentKVCache(1, 0, device="cpu")
    c = LatentKVCache(2, 16, device="cpu")
    assert c.current_len == 0 and c.remaining_capacity == 16
    assert c.kv_latent.shape == (2, 16, 512) and c.k_pe_cache.shape == (2, 16, 64)
    assert c.memory_bytes == (2 * 16 * 576) * 2
    assert c.rstd is None and c.side_bytes == 0


def test_update_get_reset_and_overflow():
    c = LatentKVCache(2, 10, device="cpu")
    a = torch.randn(2, 4, 512)
    k = torch.randn(2, 4, 64)
    c.update(a, k)
    c.update(a[:, :3], k[:, :3])
    assert c.current_len == 7 and c.remaining_capacity == 3
    lat, kpe = c.get()
    assert lat.shape == (2, 7, 512) and kpe.shape == (2, 7, 64)
    assert torch.equal(lat[:, :4], a.to(torch.bfloat16)) and torch.equal(kpe[:, 4:], k[:, :3].to(torch.bfloat16))
    assert lat.data_ptr() == c.kv_latent.data_ptr()  # zero-copy view
    assert c.get(2)[0].shape == (2, 2, 512)
    with pytest.raises(ValueError, match="Requested seq_len=8 but cache only has 7 tokens"):
        c.get(8)
    with pytest.raises(RuntimeError, match="KV cache overflow"):
        c.update(a, k)
    with pytest.raises(ValueError, match="compressed_kv must be 3D"):
        c.update(a[0], k)
    with pytest.raises(ValueError, match="k_pe must be 3D"):
        c.update(a, k[0])
    c.reset()
    assert c.current_len == 0 and c.remaining_capacity == 10
    assert "tokens=0/10" in repr(c)


def test_for_inference_defaults():
    c = LatentKVCache.for_inference(1, max_seq=64, device="cpu")
    assert c.dtype == torch.bfloat16 and c.kv_lora_rank == 512 and c.rope_head_dim == 64
    assert c.memory_bytes == 576 * 64 * 2
