"""Generate the golden fixtures that pin the CPU oracle to the reference.

    python tests/golden/make_golden.py [--reference /path/to/DeepSeek-V2-Lite-CUDA]

Runs the reference's own PyTorch code (src/reference/moe.py, src/reference/mla.py, imported
unmodified from the reference checkout; the decoder-layer residual add is restated around
the reference's RMSNorm module) on small seeded inputs and writes the inputs and
outputs to tests/golden/*.pt, together with the known answers that the reference's kernel
tests assert (tests/test_moe_scan_kernel.py, tests/test_moe_combine_kernel.py,
tests/test_moe_routing_kernel.py).  The reference is only needed to regenerate the files;
the tests read the committed fixtures.
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference(root: str):
    sys.path.insert(0, os.path.join(root, "src"))
    from reference import moe as ref_moe  # noqa: E402
    from reference import mla as ref_mla  # noqa: E402
    return ref_moe, ref_mla


def moe_fixture(ref_moe, name, T, H, I, E, k, n_shared, seed, x_scale=1.0, w_std=None):
    torch.manual_seed(seed)
    m = ref_moe.DeepSeekMoE(hidden_size=H, moe_intermediate_size=I, n_routed_experts=E,
                            num_experts_per_tok=k, n_shared_experts=n_shared).float().eval()
    if w_std is not None:
        with torch.no_grad():
            for p in m.parameters():
                p.normal_(0.0, w_std)
    x = torch.randn(T, H) * x_scale
    with torch.no_grad():
        out = m(x)
        logits = torch.nn.functional.linear(x, m.gate.weight)
        ref_idx, ref_w = m.gate(x)
        # tokens of each expert in the order the reference loop visits them (moe.py:90-103)
        visit = []
        for e in range(E):
            mask = ref_idx == e
            if mask.any():
                visit.append(mask.any(dim=1).nonzero().flatten())
        visit = torch.cat(visit) if visit else torch.zeros(0, dtype=torch.long)
    fx = {
        "T": T, "H": H, "I": I, "E": E, "k": k, "n_shared": n_shared,
        "x": x, "logits": logits, "out": out,
        "ref_topk_idx": ref_idx, "ref_topk_w": ref_w, "visit_order": visit,
        "gate": m.gate.weight.detach().clone(),
        "w1": torch.stack([torch.cat([ex.gate_proj.weight, ex.up_proj.weight]) for ex in m.experts]).detach(),
        "w2": torch.stack([ex.down_proj.weight for ex in m.experts]).detach(),
    }
    if m.shared_experts is not None:
        fx["shared_w1"] = torch.cat([m.shared_experts.gate_proj.weight,
                                     m.shared_experts.up_proj.weight]).detach()
        fx["shared_w2"] = m.shared_experts.down_proj.weight.detach()
    torch.save(fx, os.path.join(HERE, f"{name}.pt"))
    print(f"wrote {name}.pt  out[0,:4]={out[0, :4].tolist()}")


def mla_fixture(ref_mla, name, bsz, seq, seed, scaling_factor):
    torch.manual_seed(seed)
    norm = ref_mla.RMSNorm(512, eps=1e-6)
    with torch.no_grad():
        norm.weight.copy_(torch.rand(512) + 0.5)
    latent = torch.randn(bsz, seq, 512)
    with torch.no_grad():
        normed = norm(latent)
    rot = ref_mla.YaRNRotaryEmbedding(dim=64, max_position_embeddings=max(seq, 64), base=10000.0,
                                      scaling_factor=scaling_factor,
                                      original_max_position_embeddings=4096)
    q_pe = torch.randn(bsz, 16, seq, 64)
    k_pe = torch.randn(bsz, 1, seq, 64)
    cos, sin = rot(q_pe, seq_len=seq)
    pos = torch.arange(seq).unsqueeze(0).expand(bsz, -1)
    with torch.no_grad():
        q_rot, k_rot = ref_mla.apply_rotary_pos_emb(q_pe, k_pe, cos, sin, pos)
    w_kv = torch.randn(256, 512) * 0.02
    with torch.no_grad():
        kv_up = torch.nn.functional.linear(normed, w_kv)
    torch.save({
        "bsz": bsz, "seq": seq, "scaling_factor": scaling_factor,
        "latent": latent, "norm_weight": norm.weight.detach().clone(), "normed": normed,
        "q_pe": q_pe, "k_pe": k_pe, "cos": cos, "sin": sin, "q_rot": q_rot, "k_rot": k_rot,
        "w_kv": w_kv, "kv_up": kv_up,
    }, os.path.join(HERE, f"{name}.pt"))
    print(f"wrote {name}.pt")


def mla_forward_fixture(ref_mla, name, bsz, seq, hidden, heads, seed, scaling_factor,
                        w_std=0.05):
    """The whole DeepSeekMLA.forward (src/reference/mla.py:295-393) at reduced width (the
    per-head sizes are the real 128 + 64 / 128 and the 512-wide latent), f32 on the CPU."""
    torch.manual_seed(seed)
    m = ref_mla.DeepSeekMLA(hidden_size=hidden, num_heads=heads,
                            rope_scaling_factor=scaling_factor).float().eval()
    with torch.no_grad():
        for name_, p in m.named_parameters():
            if "layernorm" in name_:
                p.copy_(torch.rand_like(p) + 0.5)
            else:
                p.normal_(0.0, w_std)
    x = torch.randn(bsz, seq, hidden)
    with torch.no_grad():
        out = m(x)
        cos, sin = m.rotary_emb(x, seq_len=seq)
    torch.save({
        "bsz": bsz, "seq": seq, "hidden": hidden, "heads": heads,
        "scaling_factor": scaling_factor, "softmax_scale": float(m.softmax_scale),
        "x": x, "out": out, "cos": cos.clone(), "sin": sin.clone(),
        "w_q": m.q_proj.weight.detach().clone(),
        "w_kva": m.kv_a_proj_with_mqa.weight.detach().clone(),
        "norm_w": m.kv_a_layernorm.weight.detach().clone(),
        "w_kvb": m.kv_b_proj.weight.detach().clone(),
        "w_o": m.o_proj.weight.detach().clone(),
    }, os.path.join(HERE, f"{name}.pt"))
    print(f"wrote {name}.pt  out[0,0,:4]={out[0, 0, :4].tolist()}")


def decoder_glue_fixture(ref_mla, name, rows, H, seed):
    """The residual add + pre-norm of src/reference/decoder_layer.py:123-139 on bf16 hidden
    states, with the reference's RMSNorm module (src/reference/mla.py:53-64)."""
    torch.manual_seed(seed)
    norm = ref_mla.RMSNorm(H, eps=1e-6)
    with torch.no_grad():
        norm.weight.copy_(torch.rand(H) + 0.5)
    x = torch.randn(rows, H).to(torch.bfloat16)
    residual = (torch.randn(rows, H) * 2).to(torch.bfloat16)
    with torch.no_grad():
        summed = residual + x          # decoder_layer.py:130 / :138
        normed = norm(summed)          # decoder_layer.py:133-134 (post_attention_layernorm)
    torch.save({"x": x, "residual": residual, "weight": norm.weight.detach().clone(),
                "sum": summed, "normed": normed}, os.path.join(HERE, f"{name}.pt"))
    print(f"wrote {name}.pt")


def known_answers():
    """Known-answer cases asserted by the reference's kernel tests."""
    ka = {}
    # tests/test_moe_scan_kernel.py: random (np seed 42), zeros, single expert, uniform, skewed
    np.random.seed(42)
    rnd = np.random.randint(0, 20, size=64).astype(np.int32)
    cases = {
        "scan_random": rnd,
        "scan_zeros": np.zeros(64, dtype=np.int32),
        "scan_single": np.array([7], dtype=np.int32),
        "scan_uniform": np.full(64, 5, dtype=np.int32),
        "scan_skewed": np.concatenate([[192], np.zeros(63)]).astype(np.int32),
        "scan_sentinel": np.full(64, 3, dtype=np.int32),
    }
    for k_, c in cases.items():
        off = np.zeros(len(c) + 1, dtype=np.int32)
        off[1:] = np.cumsum(c)
        ka[k_] = (torch.from_numpy(c), torch.from_numpy(off))
    # tests/test_moe_combine_kernel.py: reference loop combine on an arbitrary-multiplicity map
    g = torch.Generator().manual_seed(7)
    T, S, H = 12, 72, 64
    eo = torch.randn(S, H, generator=g).to(torch.bfloat16)
    tm = torch.randint(0, T, (S,), generator=g, dtype=torch.int32)
    dw = torch.rand(S, generator=g)
    res = torch.zeros(T, H)
    for s in range(S):
        res[tm[s].item()] += eo[s].float() * dw[s].item()
    ka["combine"] = {"eo": eo, "token_map": tm, "dw": dw, "T": T, "out": res}
    # tests/test_moe_routing_kernel.py:155-173: all-zero logits must give k distinct experts
    ka["tie_logits"] = torch.zeros(16, 64)
    torch.save(ka, os.path.join(HERE, "known_answers.pt"))
    print("wrote known_answers.pt")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("DS_REFERENCE"),
                    help="root of a checkout of the reference project (or set DS_REFERENCE)")
    a = ap.parse_args()
    if not a.reference:
        ap.error("give --reference PATH (or set DS_REFERENCE) to the reference checkout")
    ref_moe, ref_mla = _import_reference(a.reference)
    torch.set_num_threads(4)
    # Reduced-width blocks keep the fixtures small; the algorithm is width-independent.
    moe_fixture(ref_moe, "moe_small_shared", T=24, H=64, I=32, E=8, k=2, n_shared=1, seed=0,
                w_std=0.1)
    moe_fixture(ref_moe, "moe_small_e64k6", T=40, H=32, I=16, E=64, k=6, n_shared=2, seed=1,
                w_std=0.2)
    moe_fixture(ref_moe, "moe_small_noshared", T=17, H=48, I=24, E=16, k=6, n_shared=0, seed=2,
                w_std=0.1)
    mla_fixture(ref_mla, "mla_yarn40", bsz=2, seq=16, seed=3, scaling_factor=40.0)
    mla_fixture(ref_mla, "mla_plain", bsz=1, seq=32, seed=4, scaling_factor=1.0)
    decoder_glue_fixture(ref_mla, "decoder_glue", rows=12, H=256, seed=5)
    mla_forward_fixture(ref_mla, "mla_forward_yarn40", bsz=2, seq=40, hidden=128, heads=2,
                        seed=6, scaling_factor=40.0)
    mla_forward_fixture(ref_mla, "mla_forward_plain", bsz=1, seq=48, hidden=128, heads=3,
                        seed=7, scaling_factor=1.0)
    known_answers()


if __name__ == "__main__":
    main()
