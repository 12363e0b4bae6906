"""Failure detection on the GPU without a fault: a bounded on-device wait that nothing
completes must run out, set the device status word to DS_ERR_TIMEOUT and return, leaving
the context usable for the next op."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives():
    import ds_kernels
    ds_kernels.clear_device_status()
    assert ds_kernels.device_status() == ds_kernels.DS_OK
    ds_kernels.debug_wait_probe(2_000_000)  # ~1 ms of SM clocks
    assert ds_kernels.device_status() == ds_kernels.DS_ERR_TIMEOUT
    ds_kernels.clear_device_status()
    assert ds_kernels.device_status() == ds_kernels.DS_OK
    # the context still works
    logits = torch.randn(8, 64).cuda()
    idx, w, counts = ds_kernels.moe_routing(logits, top_k=6)
    assert int(counts.sum()) == 48


def test_hello_runs():
    import ds_kernels
    ds_kernels.run_hello()
