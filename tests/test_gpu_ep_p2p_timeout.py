"""Bounded waits of the peer-memory exchange (two GPUs).

The peer path synchronises the ranks with epoch flags that each rank's
kernels poll in their peers' windows.  A rank that leaves makes the other
rank's wait run out: here rank 1 simply skips one layer call (made on the
host, between calls, with none of its kernels in flight), so rank 0's pull
kernel polls a flag that nothing sets.  The wait gives up after the
communicator's timeout, the next har_cuda_synchronize returns
HAR_CUDA_ERR_TIMEOUT, and the context stays usable.  No fault, trap or
endless loop: the kernel returns and the host reads the status.  Runs as two
child processes, one per GPU, with NVLS off; skipped with fewer than two GPUs.
"""
import os
import socket
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
mp = pytest.importorskip("torch.multiprocessing")

import har_cuda  # noqa: E402

E, H, I, K, T = 8, 512, 256, 2, 8
TIMEOUT_MS = 1500


def worker(rank, world, port, q):
    try:
        import datetime

        import haro
        import torch.distributed as dist

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120))
        ctx = har_cuda.Context(rank)
        box = [har_cuda.ep_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        ep = ctx.ep_create(box[0], world, rank, timeout_ms=TIMEOUT_MS)
        ep.set_p2p(True)
        lo, hi = har_cuda.expert_range(E, world, rank)
        El = hi - lo

        def gen(rows, k_dim, seed):
            t = torch.empty(rows * (k_dim // 256) * 144, dtype=torch.uint8, device=dev)
            ctx.gen_q4k(t, rows, k_dim, seed)
            return t

        rb_h, rb_i = H // 256 * 144, I // 256 * 144
        dg, du, dd = gen(E * I, H, 1), gen(E * I, H, 2), gen(E * H, I, 3)
        local = ctx.moe_layer(ctx.wrap_q4k(dg[lo * I * rb_h:hi * I * rb_h], El, I, H),
                              ctx.wrap_q4k(du[lo * I * rb_h:hi * I * rb_h], El, I, H),
                              ctx.wrap_q4k(dd[lo * H * rb_i:hi * H * rb_i], El, H, I))
        x = torch.from_numpy(haro.normal_f32(40 + rank, 0, T * H).reshape(T, H)).to(dev)
        ids_np, w_np = haro.zipf_routing(50 + rank, T, E, K)
        ids = torch.from_numpy(ids_np).to(dev)
        w = torch.from_numpy(w_np).to(dev)
        y = torch.empty_like(x)
        flags = har_cuda.MOE_ADD_RESIDUAL
        # one call on both ranks: maps the windows
        ctx.ep_moe_ffn(ep, local, None, None, x, ids, w, y, flags)
        torch.cuda.synchronize()
        ctx.synchronize()
        mode = ep.exchange_mode
        dist.barrier()
        info = {"mode": mode}
        if mode == 1:
            if rank == 0:
                # rank 1 does not take part in this call
                t0 = time.monotonic()
                ctx.ep_moe_ffn(ep, local, None, None, x, ids, w, y, flags)
                torch.cuda.synchronize()
                status = None
                try:
                    ctx.synchronize()
                except har_cuda.HarCudaError as e:
                    status = e.status
                info["elapsed"] = time.monotonic() - t0
                info["status"] = status
                # the context is still usable
                z = torch.ones(16, device=dev)
                info["ctx_ok"] = float(z.sum()) == 16.0
            dist.barrier()
            ep.abort()  # both ranks learn of the failure on the host and drop the exchange
        dist.barrier()
        ep.free()
        dist.destroy_process_group()
        q.put((rank, "ok", info))
    except Exception as e:  # report to the parent instead of hanging it
        import traceback
        q.put((rank, "fail", traceback.format_exc() + str(e)))


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.timeout(300)
def test_peer_wait_times_out_when_a_rank_skips_a_layer():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = []
    try:
        for _ in procs:
            results.append(q.get(timeout=240))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    by_rank = {}
    for rank, status, info in results:
        assert status == "ok", f"rank {rank}: {info}"
        by_rank[rank] = info
    if by_rank[0]["mode"] != 1:
        pytest.skip("the windows could not be mapped on this box (NCCL path only)")
    r0 = by_rank[0]
    assert r0["status"] == har_cuda.ERR_TIMEOUT, r0
    assert 1.0 < r0["elapsed"] < 30.0, r0
    assert r0["ctx_ok"], r0
