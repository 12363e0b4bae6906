"""CPU oracle for the DeepSeek-V2-Lite MoE layer and MLA projection path.

TEST INFRASTRUCTURE ONLY.  This package restates, on the CPU in float32, the algorithms of
the reference project (sahan974/DeepSeek-V2-Lite-CUDA) for the ops that
libds_kernels_sm100.so implements.  It is the checker: only tests/, __graft_entry__.smoke()
and bench.py (cpu_baseline and --impl reference) may import it.  The product path
(deepseek-v2-lite-cuda_b200/) never imports, calls or falls back to it.

Pinning: tests/test_oracle_golden.py checks every function here against golden vectors that
tests/golden/make_golden.py produced by running the reference's own PyTorch code
(src/reference/moe.py, src/reference/mla.py) and its test-file known answers.
"""
from .moe_oracle import (  # noqa: F401
    route, expert_counts, expert_offsets, dispatch, combine, swiglu, grouped_linear,
    moe_forward, MoEWeights, make_moe_weights, zipf_logits, dense_mlp,
)
from .mla_oracle import (  # noqa: F401
    rms_norm, rms_norm_residual, rope, yarn_cos_sin, kv_upproj, mla_attention, mla_forward,
    mla_forward_rows, mla_decode_step,
)
