"""Error behaviour of the drop-in op surface (runs on CPU, no GPU needed): every op rejects
bad tensors before any launch with the same RuntimeError message as the reference binding's
first failing TORCH_CHECK (src/kernels/moe/{routing,scan,dispatch,combine,gemm1,gemm2,
swiglu}.cu, src/kernels/mla/{rms_norm,kv_upproj,rope}.cu), so callers that match on those
messages keep working."""
import pytest
import torch


def ds():
    import ds_kernels
    return ds_kernels


bf = torch.bfloat16
i32 = torch.int32

# op -> (call with CPU tensors, the reference's message for a non-CUDA input)
CPU_INPUT = {
    "moe_routing": (lambda d: d.moe_routing(torch.zeros(4, 64), top_k=6),
                    "Input logits must reside on a CUDA device."),
    "moe_scan": (lambda d: d.moe_scan(torch.zeros(64, dtype=i32)),
                 "Input expert_counts must reside on a CUDA device."),
    "moe_dispatch": (lambda d: d.moe_dispatch(torch.zeros(4, 64, dtype=bf),
                                              torch.zeros(4, 6, dtype=i32), torch.zeros(4, 6),
                                              torch.zeros(65, dtype=i32)),
                     "input must reside on a CUDA device."),
    "moe_combine": (lambda d: d.moe_combine(torch.zeros(24, 64, dtype=bf),
                                            torch.zeros(24, dtype=i32), torch.zeros(24), 4),
                    "expert_output must reside on a CUDA device."),
    "moe_gemm1": (lambda d: d.moe_gemm1(torch.zeros(24, 64, dtype=bf),
                                        torch.zeros(2, 256, 64, dtype=bf),
                                        torch.zeros(3, dtype=i32)),
                  "gemm1: dispatched must be a contiguous CUDA tensor."),
    "moe_gemm2": (lambda d: d.moe_gemm2(torch.zeros(24, 128, dtype=bf),
                                        torch.zeros(2, 64, 128, dtype=bf),
                                        torch.zeros(3, dtype=i32)),
                  "gemm2: swiglu_out must be a contiguous CUDA tensor."),
    "swiglu": (lambda d: d.swiglu(torch.zeros(4, 256, dtype=bf)),
               "swiglu: input must be a CUDA tensor."),
    "rms_norm": (lambda d: d.rms_norm(torch.zeros(4, 512, dtype=bf), torch.ones(512)),
                 "rms_norm: input must be a CUDA tensor."),
    "kv_upproj": (lambda d: d.kv_upproj(torch.zeros(4, 512, dtype=bf),
                                        torch.zeros(4096, 512, dtype=bf)),
                  "kv_upproj: normed_kv must be a contiguous CUDA tensor."),
    "rope": (lambda d: d.rope(torch.zeros(1, 2, 4, 64, dtype=bf), torch.zeros(1, 1, 4, 64, dtype=bf),
                              torch.zeros(1, 1, 4, 64, dtype=bf), torch.zeros(1, 1, 4, 64, dtype=bf)),
             "rope: all inputs must be contiguous CUDA tensors."),
}


@pytest.mark.parametrize("op", sorted(CPU_INPUT))
def test_cpu_input_rejected_with_reference_message(op):
    call, msg = CPU_INPUT[op]
    with pytest.raises(RuntimeError) as e:
        call(ds())
    assert str(e.value) == msg


def test_c_abi_reports_bad_arguments_without_a_gpu():
    # the C ABI validates shapes before touching the device: a bad top_k comes back as
    # DS_ERR_INVALID_ARG with a message, no launch and no device needed
    d = ds()
    lib = d.library()
    st = lib.ds_moe_routing(None, None, None, None, 4, 64, 9, None)
    assert st == d.DS_ERR_INVALID_ARG
    assert lib.ds_last_error().decode()
