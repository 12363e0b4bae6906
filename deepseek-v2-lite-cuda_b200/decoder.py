"""DeepSeek-V2-Lite decoder stack on the fused kernels (configs 3 and 4).

One layer is the pre-norm block of src/reference/decoder_layer.py:123-139:

    h = x + attn(RMSNorm_in(x));   out = h + ffn(RMSNorm_post(h))

with attn = mla.FusedMLA (prefill over a prompt, or decode of one token per sequence over a
latent KV cache), ffn = moe_fused.FusedMoELayer for layers 1-26 and the dense SwiGLU
2048 -> 10944 -> 2048 for layer 0 (first_k_dense_replace = 1, decoder_layer.py:8-9).  Every
residual add is fused with the RMSNorm that follows it (ds_rms_norm_residual: the bf16 sum
and its norm in one pass), so a layer is: MLA, norm+add, FFN, norm+add.
"""
from __future__ import annotations

import math
from typing import List, Optional, Sequence

import torch

import ds_kernels
from mla import FusedMLA
from mla_cache import LatentKVCache


class DenseFFN:
    """Layer 0's dense SwiGLU FFN: w1 = [gate; up] bf16 [2I, H], w2 bf16 [H, I]."""

    def __init__(self, w1: torch.Tensor, w2: torch.Tensor):
        self.w1, self.w2 = w1.contiguous(), w2.contiguous()
        self._ws: Optional[torch.Tensor] = None

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        # few rows (decode): the GEMMs split K over the SMs (workspace grown once)
        need = int(ds_kernels.library().ds_dense_mlp_workspace_size(
            x.shape[0], self.w1.shape[1], self.w1.shape[0] // 2))
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(max(need, 1), dtype=torch.uint8, device=x.device)
        return ds_kernels.dense_mlp_ws(x, self.w1, self.w2, workspace=self._ws)


class FusedDecoderLayer:
    def __init__(self, attn: FusedMLA, ffn, w_in: torch.Tensor, w_post: torch.Tensor,
                 eps: float = 1e-6):
        self.attn, self.ffn = attn, ffn
        self.w_in = w_in.detach().float().contiguous()
        self.w_post = w_post.detach().float().contiguous()
        self.eps = eps


class FusedDecoderStack:
    """A stack of FusedDecoderLayer; prefill() fills one LatentKVCache per layer, decode_step()
    runs one token per sequence through every layer."""

    def __init__(self, layers: Sequence[FusedDecoderLayer]):
        self.layers = list(layers)

    def new_caches(self, bsz: int, max_seq: int, device=None) -> List[LatentKVCache]:
        dev = device if device is not None else self.layers[0].w_in.device
        return [LatentKVCache(bsz, max_seq, device=dev) for _ in self.layers]

    def _run(self, x2: torch.Tensor, attn_fn, ffn_rows) -> torch.Tensor:
        L = self.layers
        eps = L[0].eps
        hidden = x2
        normed = ds_kernels.rms_norm(hidden, L[0].w_in, eps)
        for i, layer in enumerate(L):
            a = attn_fn(layer, normed, i)
            normed2, hidden = ds_kernels.rms_norm_residual(a, hidden, layer.w_post, layer.eps)
            f = layer.ffn(ffn_rows(normed2))
            f = f.view(hidden.shape)
            w_next = L[i + 1].w_in if i + 1 < len(L) else layer.w_in
            normed, hidden = ds_kernels.rms_norm_residual(f, hidden, w_next, eps)
        return hidden

    def decode_step(self, x: torch.Tensor, caches: Sequence[LatentKVCache]) -> torch.Tensor:
        """x bf16 [bsz, hidden] (one new token per sequence) -> [bsz, hidden]."""
        return self._run(x.contiguous(), lambda layer, h, i: layer.attn.decode(h, caches[i]),
                         lambda h: h)

    def capture_decode(self, x: torch.Tensor, caches: Sequence[LatentKVCache]) -> torch.Tensor:
        """Run one decode step eagerly (it allocates the workspaces and brings the caches' side
        arrays up to date, and advances the caches by one position), then record the step as a
        CUDA graph: the ~15 launches of each of the layers become one graph launch.  The
        kernels read the position from each cache's device-side length and advance it, so
        replay_decode() steps through successive positions.  Returns the eager step's output."""
        self._graph_x = x.contiguous().clone()
        first = self.decode_step(self._graph_x, caches)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            with torch.cuda.graph(graph, stream=stream):
                self._graph_out = self.decode_step(self._graph_x, caches)
        torch.cuda.current_stream().wait_stream(stream)
        # recording ran the host-side bookkeeping of one step without executing it on the GPU
        for c in caches:
            c._len -= 1
            c._side_len -= 1
        self._graph = graph
        self._graph_caches = list(caches)
        return first

    def replay_decode(self, x: torch.Tensor) -> torch.Tensor:
        """One decode step through the captured graph: x bf16 [bsz, hidden] is copied into the
        graph's input; returns the graph's output buffer (overwritten by the next replay)."""
        for c in self._graph_caches:
            if c.current_len >= c.max_seq:
                raise RuntimeError("replay_decode: a cache is full")
        self._graph_x.copy_(x, non_blocking=True)
        self._graph.replay()
        for c in self._graph_caches:
            c._len += 1
            c._side_len += 1
        return self._graph_out

    def prefill(self, x: torch.Tensor, caches: Sequence[LatentKVCache]) -> torch.Tensor:
        """x bf16 [bsz, seq, hidden] (prompts at positions 0 .. seq-1) -> [bsz, seq, hidden];
        fills the caches."""
        B, S, H = x.shape
        return self._run(x.contiguous(),
                         lambda layer, h, i: layer.attn.prefill(h, caches[i]),
                         lambda h: h.view(B * S, H))


def yarn_tables(positions: int, scaling_factor: float, device, dim: int = 64,
                base: float = 10000.0, original_max: int = 4096, beta_fast: float = 32,
                beta_slow: float = 1, mscale: float = 0.707, mscale_all_dim: float = 0.707):
    """bf16 cos/sin [positions, 64] with DeepSeek-V2-Lite's YaRN RoPE (scaling_factor 1 gives
    plain RoPE with theta = base), the tables of src/reference/mla.py:66-173, and the softmax
    scale 192^-0.5 * mscale^2 of mla.py:292-293."""
    def corr(n_rot):
        return (dim * math.log(original_max / (n_rot * 2 * math.pi))) / (2 * math.log(base))

    def msc(scale, m):
        return 1.0 if scale <= 1 else 0.1 * m * math.log(scale) + 1.0
    pos_freq = base ** (torch.arange(0, dim, 2, dtype=torch.float32, device=device) / dim)
    lo = max(math.floor(corr(beta_fast)), 0)
    hi = min(math.ceil(corr(beta_slow)), dim - 1)
    if lo == hi:
        hi += 0.001
    ramp = torch.clamp((torch.arange(dim // 2, dtype=torch.float32, device=device) - lo) / (hi - lo), 0, 1)
    inv = (1.0 / (scaling_factor * pos_freq)) * ramp + (1.0 / pos_freq) * (1.0 - ramp)
    t = torch.arange(positions, dtype=torch.float32, device=device)
    emb = torch.cat([torch.outer(t, inv)] * 2, dim=-1)
    m = msc(scaling_factor, mscale) / msc(scaling_factor, mscale_all_dim)
    ms = msc(scaling_factor, mscale_all_dim)
    return ((emb.cos() * m).to(torch.bfloat16), (emb.sin() * m).to(torch.bfloat16),
            192 ** -0.5 * ms * ms)


def random_stack(n_layers: int, device, hidden: int = 2048, heads: int = 16,
                 dense_inter: int = 10944, moe_inter: int = 1408, experts: int = 64,
                 top_k: int = 6, n_shared: int = 2, positions: int = 4096,
                 scaling_factor: float = 40.0, std: float = 0.02, seed: int = 0,
                 first_dense: int = 1) -> FusedDecoderStack:
    """Random-init weights of the DeepSeek-V2-Lite architecture (N(0, std^2); norm weights 1):
    layers [0, first_dense) dense FFN, the rest MoE.  Generated on `device`, layer by layer."""
    from moe_fused import FusedMoELayer
    import synthetic
    g = torch.Generator(device=device).manual_seed(seed)
    cos, sin, scale = yarn_tables(positions, scaling_factor, device)

    def w(*shape):
        return (torch.randn(*shape, generator=g, device=device) * std).to(torch.bfloat16)

    layers = []
    for i in range(n_layers):
        attn = FusedMLA.from_weights(w(heads * 192, hidden), w(576, hidden),
                                     torch.ones(512, device=device), w(heads * 256, 512),
                                     w(hidden, heads * 128), cos, sin, scale, heads)
        if i < first_dense:
            ffn = DenseFFN(w(2 * dense_inter, hidden), w(hidden, dense_inter))
        else:
            W = synthetic.make_layer_weights(seed * 1000 + i, device, hidden, moe_inter, experts,
                                             n_shared, std)
            ffn = FusedMoELayer.from_packed(W.gate, W.packed_w1, W.w2, W.shared_w1, W.shared_w2,
                                            top_k=top_k)
        layers.append(FusedDecoderLayer(attn, ffn, torch.ones(hidden, device=device),
                                        torch.ones(hidden, device=device)))
    return FusedDecoderStack(layers)
