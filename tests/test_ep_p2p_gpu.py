"""Expert parallelism over NVLink peer memory (ep_p2p.P2PEPMoELayer -> ds_ep_layer_forward).

Every routed row is computed by the same kernels as on one GPU and combined in the same
slot order, so the expert-parallel output must equal the single-GPU fused layer
(moe_fused.FusedMoELayer, itself checked against the CPU oracle) bit for bit; one case is
also checked against the oracle directly (max-abs 2e-2, rel-L2 1e-2).  Failure detection:
a rank that stops taking part makes the other rank's bounded in-kernel wait run out; the
device status reads DS_ERR_TIMEOUT and the context stays usable.  Multi-rank cases run one
process per GPU (2, 4 and 8 ranks, each skipped without enough GPUs), NVLS off, plain peer
loads and stores.
"""
import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

H, I, E, K = 2048, 1408, 64, 6


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layers(seed, dev, rank, world, max_tokens, timeout_ms=10000):
    import synthetic
    from ep_p2p import P2PEPMoELayer
    from moe_fused import FusedMoELayer
    W = synthetic.make_layer_weights(seed, dev)
    ref = FusedMoELayer.from_packed(W.gate, W.packed_w1, W.w2, W.shared_w1, W.shared_w2, top_k=K)
    El = E // world
    ep = P2PEPMoELayer(W.gate, W.packed_w1[rank * El:(rank + 1) * El].clone(),
                       W.w2[rank * El:(rank + 1) * El].clone(), W.shared_w1, W.shared_w2,
                       top_k=K, max_tokens=max_tokens, timeout_ms=timeout_ms)
    return W, ref, ep


def test_one_rank_equals_fused_layer():
    import ds_kernels
    import synthetic
    ds_kernels.clear_device_status()
    dev = torch.device("cuda:0")
    _, ref, ep = _layers(31, dev, 0, 1, 4096)
    try:
        for i, T in enumerate((1, 300, 0, 4096, 129)):
            x = synthetic.make_tokens(100 + i, T, H, dev)
            lg = torch.empty(T, E, device=dev)
            lg_ref = torch.empty(T, E, device=dev)
            out = ep(x, logits_out=lg)
            want = ref(x, logits_out=lg_ref)
            assert out.shape == (T, H)
            assert torch.equal(out, want), T
            assert torch.equal(lg, lg_ref), T
        ep.check()
    finally:
        ep.close()


def test_one_rank_host_pipeline_writes_into_slot_outputs():
    # HostPipeline hands the layer its per-slot output buffers (out=); the pipelined results
    # must equal direct calls bit for bit, and the layer must write into the buffer it got
    import ds_kernels
    import synthetic
    from moe_fused import HostPipeline
    ds_kernels.clear_device_status()
    dev = torch.device("cuda:0")
    _, ref, ep = _layers(33, dev, 0, 1, 1024)
    try:
        xs = [synthetic.make_tokens(200 + i, T, H, dev).cpu().pin_memory()
              for i, T in enumerate((1024, 17, 512, 1024, 1))]
        outs = [torch.empty(x.shape, dtype=torch.bfloat16).pin_memory() for x in xs]
        pipe = HostPipeline(ep, max_tokens=1024, hidden=H)
        assert pipe.takes_out
        for x, o in zip(xs, outs):
            pipe.submit(x, o)
        pipe.synchronize()
        for x, o in zip(xs, outs):
            assert torch.equal(o, ref(x.to(dev)).cpu())
        buf = torch.empty(300, H, dtype=torch.bfloat16, device=dev)
        x = synthetic.make_tokens(9, 300, H, dev)
        assert ep(x, out=buf).data_ptr() == buf.data_ptr()
        assert torch.equal(buf, ref(x))
        ep.check()
    finally:
        ep.close()


def test_one_rank_matches_oracle():
    import ds_kernels
    import oracle
    from conftest import assert_bf16_close
    from ep_p2p import P2PEPMoELayer
    ds_kernels.clear_device_status()
    dev = torch.device("cuda:0")
    W = oracle.make_moe_weights(9, H, I, E, n_shared=2)
    g = torch.Generator().manual_seed(10)
    x = torch.randn(200, H, generator=g).to(torch.bfloat16)
    ep = P2PEPMoELayer(W.gate.to(dev), W.w1.to(torch.bfloat16).to(dev),
                       W.w2.to(torch.bfloat16).to(dev), W.shared_w1.to(torch.bfloat16).to(dev),
                       W.shared_w2.to(torch.bfloat16).to(dev), top_k=K, max_tokens=256)
    try:
        lg = torch.empty(200, E, device=dev)
        out = ep(x.to(dev), logits_out=lg)
        ref = oracle.moe_forward(x, W, K, logits=lg.cpu())
        assert_bf16_close(out, ref, 2e-2)
        ep.check()
    finally:
        ep.close()


def test_one_rank_wait_times_out_and_context_survives():
    # the count exchange waits for a forward number nothing ever reaches: the bounded wait
    # runs out (50 ms), the status word reads DS_ERR_TIMEOUT, later kernels skip their waits
    import ds_kernels
    import synthetic
    ds_kernels.clear_device_status()
    dev = torch.device("cuda:0")
    _, ref, ep = _layers(32, dev, 0, 1, 512, timeout_ms=50)
    x = synthetic.make_tokens(7, 256, H, dev)
    try:
        assert torch.equal(ep(x), ref(x))
        ep.check()
        ep._epoch += 2  # skew the forward number: the flags never reach the new target
        ep(x)
        with pytest.raises(RuntimeError, match="cross-GPU wait"):
            ep.check()
        assert ds_kernels.device_status() == ds_kernels.DS_ERR_TIMEOUT
    finally:
        ds_kernels.clear_device_status()
        ep.close()
    # the context is still usable: a fresh layer computes the right answer
    _, ref2, ep2 = _layers(32, dev, 0, 1, 512)
    try:
        assert torch.equal(ep2(x), ref2(x))
        ep2.check()
    finally:
        ep2.close()


def _worker(rank, world, port, mode, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "deepseek-v2-lite-cuda_b200"))
    sys.path.insert(0, root)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        import torch.distributed as dist
        import ds_kernels
        import synthetic
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=120))
        ds_kernels.clear_device_status()
        result = None
        if mode == "exact":
            _, ref, ep = _layers(41, dev, rank, world, 4096)
            sizes = [(300, 4096), (4096, 1), (0, 129), (17, 0), (4096, 4096)]
            ok = []
            for i, ts in enumerate(sizes):
                T = ts[rank % 2]
                x = synthetic.make_tokens(1000 * rank + i, T, H, dev)
                out = ep(x)
                again = ref(x)
                ok.append(bool(torch.equal(out, again)))
            ep.check()
            result = ok
        else:  # "leave": rank 1 stops taking part after the first forward
            _, ref, ep = _layers(42, dev, rank, world, 512, timeout_ms=200)
            x = synthetic.make_tokens(5 + rank, 256, H, dev)
            first = bool(torch.equal(ep(x), ref(x)))
            ep.check()
            dist.barrier(device_ids=[rank])
            status = None
            if rank == 0:
                ep(x)  # its peer never joins this forward
                try:
                    ep.check()
                    status = "no error"
                except RuntimeError:
                    status = ds_kernels.device_status()
                ds_kernels.clear_device_status()
            dist.barrier(device_ids=[rank])
            result = (first, status)
        ep.close()
        dist.destroy_process_group()
        q.put((rank, result, None))
    except Exception as e:  # noqa: BLE001
        q.put((rank, None, repr(e)))


def _run(world, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=900) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    return sorted(res)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ranks_equal_fused_layer(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    for rank, ok, exc in _run(world, "exact"):
        assert exc is None, (rank, exc)
        assert all(ok), (rank, ok)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_ranks_peer_leaves_wait_times_out():
    import ds_kernels
    res = _run(2, "leave")
    for rank, r, exc in res:
        assert exc is None, (rank, exc)
        assert r[0], rank
    assert res[0][1][1] == ds_kernels.DS_ERR_TIMEOUT
