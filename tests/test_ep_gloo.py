"""Expert-parallel orchestration (ep_moe.EPMoELayer) on CPU ranks with the gloo backend.

The layer's compute steps are replaced by an oracle-backed CPU implementation, so these
tests exercise the host logic of the N > 1 path: expert sharding, the counts exchange, the
split sizes, the row all-to-alls, the receive-side plan (expert-major offsets and row map)
and the return path into the token owners' slot order.  Every rank's output must equal the
single-process oracle MoE forward on the same tokens.  A second test makes one rank leave
before the exchange and checks that its peer fails within the short process-group timeout
instead of hanging.
"""
import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

H, I, E, K = 64, 32, 8, 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class CpuOps:
    """f32 CPU stand-in for CudaOps, built on the oracle."""

    def prepare_router(self, gate):
        return gate.float()

    def route(self, x, gate, num_experts, top_k):
        import oracle
        return oracle.route(x.float() @ gate.t(), top_k)

    def dispatch(self, idx, w, x, num_experts):
        import oracle
        disp, tmap, dw, slot_of, off = oracle.dispatch(x, idx, w, num_experts)
        return off, slot_of, tmap, disp.contiguous()

    def ep_plan(self, recv_counts, R):
        N, El = recv_counts.shape
        c = recv_counts.long()
        seg_src = torch.cumsum(c.reshape(-1), 0) - c.reshape(-1)
        off = torch.zeros(El + 1, dtype=torch.long)
        off[1:] = torch.cumsum(c.sum(0), 0)
        row_map = torch.empty(R, dtype=torch.long)
        for e in range(El):
            pos = int(off[e])
            for s in range(N):
                n = int(c[s, e])
                src0 = int(seg_src[s * El + e])
                row_map[pos:pos + n] = torch.arange(src0, src0 + n)
                pos += n
        return off.to(torch.int32), row_map.to(torch.int32)

    def gather_rows(self, src, row_map):
        return src[row_map.long()]

    def expert_mlp(self, rows, offsets, w1, w2, out, out_row_map):
        from oracle.moe_oracle import _mlp
        off = offsets.tolist()
        for e in range(w1.shape[0]):
            a, b = off[e], off[e + 1]
            if b > a:
                out[out_row_map[a:b].long()] = _mlp(rows[a:b].float(), w1[e].float(), w2[e].float())
        return out

    def dense_mlp(self, x, w1, w2, max_ctas=0):
        from oracle.moe_oracle import _mlp
        return _mlp(x.float(), w1.float(), w2.float())

    def shared_gemm1(self, x, w1, max_ctas=0):
        I = w1.shape[0] // 2
        h = x.float() @ w1.float().t()
        g, u = h[:, :I], h[:, I:]
        return g / (1.0 + torch.exp(-g)) * u

    def shared_gemm2(self, h, w2, max_ctas=0):
        return h @ w2.float().t()

    def num_sms(self, device):
        return 0

    def combine_slots(self, back, slot_of, w, shared_out):
        T, k = slot_of.shape
        out = torch.zeros(T, back.shape[1])
        order = torch.argsort(slot_of.long(), dim=1)
        for j in range(k):
            sel = torch.gather(slot_of.long(), 1, order[:, j:j + 1]).squeeze(1)
            ww = torch.gather(w, 1, order[:, j:j + 1])
            out += back[sel].float() * ww
        if shared_out is not None:
            out += shared_out.float()
        return out


def _worker(rank, world, port, T_per_rank, q, n_shared):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "deepseek-v2-lite-cuda_b200"))
    sys.path.insert(0, root)
    import torch.distributed as dist
    import oracle
    from ep_moe import EPMoELayer, shard_experts
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        W = oracle.make_moe_weights(5, H=H, I=I, E=E, n_shared=n_shared, std=0.2, round_bf16=False)
        g = torch.Generator().manual_seed(9)
        x_all = torch.randn(T_per_rank * world, H, generator=g)
        x = x_all[rank * T_per_rank:(rank + 1) * T_per_rank].contiguous()
        w1, w2 = shard_experts(W.w1, W.w2, rank, world)
        layer = EPMoELayer(W.gate, w1, w2, W.shared_w1, W.shared_w2, top_k=K, ops=CpuOps())
        out = layer(x)
        ref = oracle.moe_forward(x_all, W, K)[rank * T_per_rank:(rank + 1) * T_per_rank]
        err = (out - ref).abs().max().item()
        dist.destroy_process_group()
        q.put((rank, err, None))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, None, repr(e)))


def _run(world, T_per_rank, n_shared):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, T_per_rank, q, n_shared))
             for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    return res


@pytest.mark.parametrize("world,T,n_shared", [(2, 37, 1), (4, 20, 0), (2, 1, 1)])
def test_ep_layer_matches_single_process_oracle(world, T, n_shared):
    for rank, err, exc in _run(world, T, n_shared):
        assert exc is None, (rank, exc)
        assert err <= 1e-4, (rank, err)


def _leaver(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        q.put((rank, "left"))
        q.close()
        q.join_thread()  # flush the message before leaving
        os._exit(0)  # leaves between steps, before the exchange
    t = torch.zeros(2, dtype=torch.int32)
    o = torch.empty_like(t)
    import time
    t0 = time.time()
    try:
        dist.all_to_all_single(o, t)
        q.put((rank, "no error"))
    except Exception as e:
        q.put((rank, f"error after {time.time() - t0:.1f}s: {type(e).__name__}"))


def test_peer_leaving_is_detected_not_hung():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaver, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert res[1] == "left"
    assert res[0].startswith("error"), res[0]
