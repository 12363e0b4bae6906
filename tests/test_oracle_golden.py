"""Pin the CPU oracle to the reference: every oracle function against the golden vectors that
tests/golden/make_golden.py produced by running the reference's own PyTorch code, and the
known answers of the reference's kernel tests.  CPU only."""
import os
import pytest

import torch

import oracle
from oracle.moe_oracle import MoEWeights

from conftest import GOLDEN


def _load(name):
    return torch.load(os.path.join(GOLDEN, name), weights_only=False)


def _weights(fx):
    return MoEWeights(fx["gate"], fx["w1"], fx["w2"], fx.get("shared_w1"), fx.get("shared_w2"))


def _check_moe(name):
    fx = _load(name)
    out = oracle.moe_forward(fx["x"], _weights(fx), fx["k"])
    # f32 on both sides; only summation order differs
    torch.testing.assert_close(out, fx["out"], atol=2e-5, rtol=1e-5)
    # routing: same expert SET per token and same weights as MoEGate (topk(sorted=False))
    idx, w = oracle.route(fx["logits"], fx["k"])
    ref_idx, ref_w = fx["ref_topk_idx"], fx["ref_topk_w"]
    for t in range(idx.shape[0]):
        assert set(idx[t].tolist()) == set(ref_idx[t].tolist()), t
    full = torch.zeros(idx.shape[0], fx["E"]).scatter_(1, idx.long(), w)
    ref_full = torch.zeros(idx.shape[0], fx["E"]).scatter_(1, ref_idx.long(), ref_w)
    torch.testing.assert_close(full, ref_full, atol=1e-6, rtol=0)
    # permutation: expert-major, tokens in the order the reference loop visits them
    _, token_map, _, slot_of, offsets = oracle.dispatch(fx["x"], idx, w, fx["E"])
    assert torch.equal(token_map.long(), fx["visit_order"])
    counts = oracle.expert_counts(idx, fx["E"])
    assert int(offsets[-1]) == fx["T"] * fx["k"] == int(counts.sum())


def test_moe_forward_small_shared():
    _check_moe("moe_small_shared.pt")


def test_moe_forward_e64_k6():
    _check_moe("moe_small_e64k6.pt")


def test_moe_forward_no_shared():
    _check_moe("moe_small_noshared.pt")


def test_dispatch_slot_of_inverts_token_map():
    fx = _load("moe_small_e64k6.pt")
    idx, w = oracle.route(fx["logits"], fx["k"])
    dispatched, token_map, dw, slot_of, offsets = oracle.dispatch(fx["x"], idx, w, fx["E"])
    T, k = idx.shape
    for t in range(T):
        for j in range(k):
            s = int(slot_of[t, j])
            assert int(token_map[s]) == t
            assert float(dw[s]) == float(w[t, j])
            e = int(idx[t, j])
            assert int(offsets[e]) <= s < int(offsets[e + 1])
            assert torch.equal(dispatched[s], fx["x"][t])


def test_scan_known_answers():
    ka = _load("known_answers.pt")
    for key in ("scan_random", "scan_zeros", "scan_single", "scan_uniform", "scan_skewed",
                "scan_sentinel"):
        counts, offsets = ka[key]
        assert torch.equal(oracle.expert_offsets(counts), offsets.to(torch.int32)), key


def test_combine_known_answer():
    c = _load("known_answers.pt")["combine"]
    out = oracle.combine(c["eo"], c["token_map"], c["dw"], c["T"])
    torch.testing.assert_close(out, c["out"], atol=1e-5, rtol=1e-5)


def test_combine_zero_weights_exact_zero():
    c = _load("known_answers.pt")["combine"]
    out = oracle.combine(c["eo"], c["token_map"], torch.zeros_like(c["dw"]), c["T"])
    assert torch.all(out == 0)


def test_routing_ties_lower_index():
    logits = _load("known_answers.pt")["tie_logits"]
    idx, w = oracle.route(logits, 6)
    assert torch.equal(idx, torch.arange(6, dtype=torch.int32).expand(16, 6))
    torch.testing.assert_close(w, torch.full((16, 6), 1.0 / 64), atol=1e-7, rtol=0)


def _check_mla(name):
    fx = _load(name)
    normed = oracle.rms_norm(fx["latent"], fx["norm_weight"])
    torch.testing.assert_close(normed, fx["normed"], atol=1e-6, rtol=1e-6)
    cos, sin = oracle.yarn_cos_sin(fx["seq"], scaling_factor=fx["scaling_factor"])
    torch.testing.assert_close(cos, fx["cos"], atol=1e-6, rtol=0)
    torch.testing.assert_close(sin, fx["sin"], atol=1e-6, rtol=0)
    q_rot, k_rot = oracle.rope(fx["q_pe"], fx["k_pe"], cos[None, None], sin[None, None])
    torch.testing.assert_close(q_rot, fx["q_rot"], atol=1e-6, rtol=1e-6)
    torch.testing.assert_close(k_rot, fx["k_rot"], atol=1e-6, rtol=1e-6)
    kv = oracle.kv_upproj(fx["normed"], fx["w_kv"])
    torch.testing.assert_close(kv, fx["kv_up"], atol=1e-5, rtol=1e-5)


def test_mla_yarn40():
    _check_mla("mla_yarn40.pt")


def test_mla_plain_rope_theta():
    _check_mla("mla_plain.pt")
    # scaling_factor 1 reduces YaRN to plain RoPE with theta 10000
    cos, sin = oracle.yarn_cos_sin(8, scaling_factor=1.0)
    inv = 1.0 / (10000.0 ** (torch.arange(0, 64, 2, dtype=torch.float32) / 64))
    ang = torch.outer(torch.arange(8, dtype=torch.float32), inv)
    torch.testing.assert_close(cos, torch.cat([ang, ang], -1).cos(), atol=1e-6, rtol=0)


def test_decoder_glue_residual_rms_norm():
    # the decoder layer's residual add + RMSNorm (reference module on bf16 hidden states)
    fx = _load("decoder_glue.pt")
    normed, summed = oracle.rms_norm_residual(fx["x"], fx["residual"], fx["weight"])
    assert torch.equal(summed, fx["sum"])  # the bf16 residual sum, bit for bit
    # the reference rounds the normalised row to bf16 before the f32 weight (mla.py:64); the
    # oracle keeps it in f32 (one rounding, as the kernels do): within a bf16 half-ulp
    torch.testing.assert_close(normed, fx["normed"].float(), atol=1e-6, rtol=2.0 ** -8)


@pytest.mark.parametrize("name", ["mla_forward_yarn40.pt", "mla_forward_plain.pt"])
def test_mla_forward_matches_the_reference_module(name):
    # the whole DeepSeekMLA.forward (projections, latent RMSNorm, RoPE, causal attention with
    # 192-wide q/k and 128-wide v, o_proj), reference module run in f32 on the CPU
    fx = _load(name)
    cos, sin = oracle.yarn_cos_sin(fx["seq"], scaling_factor=fx["scaling_factor"])
    torch.testing.assert_close(cos, fx["cos"], atol=1e-6, rtol=0)
    out = oracle.mla_forward(fx["x"], fx["w_q"], fx["w_kva"], fx["norm_w"], fx["w_kvb"],
                             fx["w_o"], fx["cos"], fx["sin"], fx["softmax_scale"], fx["heads"])
    torch.testing.assert_close(out, fx["out"], atol=2e-5, rtol=2e-5)


def test_mla_forward_rows_agrees_with_the_full_forward():
    # the row-restricted oracle used to check full-length sequences on the GPU
    fx = _load("mla_forward_yarn40.pt")
    args = (fx["x"], fx["w_q"], fx["w_kva"], fx["norm_w"], fx["w_kvb"], fx["w_o"], fx["cos"],
            fx["sin"], fx["softmax_scale"], fx["heads"])
    full = oracle.mla_forward(*args)
    rows = torch.tensor([0, 1, 7, 20, 39])
    torch.testing.assert_close(oracle.mla_forward_rows(*args, rows), full[:, rows],
                               atol=1e-5, rtol=1e-5)


def test_mla_decode_step_is_the_last_row_of_the_forward():
    # the decode oracle over a cache holding a prefix's raw latents / k_pe equals the full
    # forward's row at the new position (pinned through mla_forward to the reference module)
    fx = _load("mla_forward_yarn40.pt")
    x = fx["x"]
    L = x.shape[1] - 1
    ckv = x[:, :L] @ fx["w_kva"].t()
    out = oracle.mla_decode_step(x[:, L], ckv[..., :512], ckv[..., 512:], fx["w_q"], fx["w_kva"],
                                 fx["norm_w"], fx["w_kvb"], fx["w_o"], fx["cos"], fx["sin"],
                                 fx["softmax_scale"], fx["heads"])
    full = oracle.mla_forward(x, fx["w_q"], fx["w_kva"], fx["norm_w"], fx["w_kvb"], fx["w_o"],
                              fx["cos"], fx["sin"], fx["softmax_scale"], fx["heads"])
    torch.testing.assert_close(out, full[:, L], atol=1e-5, rtol=1e-5)
