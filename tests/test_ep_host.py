"""Expert-parallel dataflow on the CPU, world size 2 over gloo.

The device path (har_cuda_ep_moe_ffn, csrc/k_ep.cu) dispatches fixed-size rows:
for every destination rank d and local token t one row with x[t] and t's k
slots as d-local expert ids (-1 where the expert lives on another rank) and
their weights; each rank computes the partial sums of the rows it receives
with its expert shard; the partial sums return to the tokens' ranks, which add
residual, the shared expert (gated by sigmoid(gate_inp . x)) and the partials.
This test restates that dataflow in numpy with the oracle's compose_moe_route
for the expert math and real all-to-alls over a two-rank gloo group, and checks
that it reproduces the unsharded layer (har-native-qwen35moe.rs:979-1048).
"""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
dist = pytest.importorskip("torch.distributed")
mp = pytest.importorskip("torch.multiprocessing")

import har_cuda  # noqa: E402

E, H, I, K, T = 8, 256, 256, 3, 5


def test_expert_range():
    assert har_cuda.expert_range(512, 8, 3) == (192, 256)
    assert har_cuda.expert_range(16, 1, 0) == (0, 16)
    with pytest.raises(ValueError):
        har_cuda.expert_range(10, 4, 0)
    with pytest.raises(ValueError):
        har_cuda.expert_range(16, 2, 2)


def plan(ids, w, G, El):
    """ep_plan_kernel's rows: [G][T][k] local ids (-1 = elsewhere) and weights."""
    owner = ids // El
    lids = np.where(owner[None, :, :] == np.arange(G)[:, None, None], ids[None] - np.arange(G)[:, None, None] * El, -1)
    lw = np.where(lids >= 0, w[None], 0.0).astype(np.float32)
    return lids.astype(np.int32), lw


def partial_sums(haro, hg, hu, hd, El, rx, rids, rw):
    """Each received row: sum over its non-empty slots of w * expert(x), slot order."""
    out = np.zeros_like(rx)
    for r in range(rx.shape[0]):
        sel = np.nonzero(rids[r] >= 0)[0]
        if len(sel) == 0:
            continue
        out[r] = haro.moe_ffn(hg, hu, hd, None, None, El, H, I, rx[r:r + 1],
                              rids[r:r + 1, sel].copy(), rw[r:r + 1, sel].copy())[0]
    return out


def worker(rank, world, port, q):
    try:
        import haro
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        El = E // world
        lo, hi = har_cuda.expert_range(E, world, rank)
        # the full layer (every rank can rebuild it: seeded generators)
        hg, hu, hd = haro.gen_q4k(11, E * I, H), haro.gen_q4k(12, E * I, H), haro.gen_q4k(13, E * H, I)
        sg, su, sd = haro.gen_q4k(14, I, H), haro.gen_q4k(15, I, H), haro.gen_q4k(16, H, I)
        gi = haro.normal_f32(17, 0, H, 0.0, 0.02)
        rb = hg.shape[1]
        # this rank's shard of the routed experts
        lg, lu = hg[lo * I:hi * I], hu[lo * I:hi * I]
        ld = hd[lo * H:hi * H]
        # this rank's tokens and routing
        x = haro.normal_f32(100 + rank, 0, T * H).reshape(T, H)
        ids, w = haro.zipf_routing(200 + rank, T, E, K)
        # 1. plan, 2. dispatch
        lids, lw = plan(ids, w, world, El)
        sx = np.broadcast_to(x, (world, T, H)).astype(np.float32).copy()
        rx, rids, rw = (torch.empty(world * T * H), torch.empty(world * T * K, dtype=torch.int32),
                        torch.empty(world * T * K))
        dist.all_to_all_single(rx, torch.from_numpy(sx.reshape(-1)))
        dist.all_to_all_single(rids, torch.from_numpy(lids.reshape(-1)))
        dist.all_to_all_single(rw, torch.from_numpy(lw.reshape(-1)))
        rx = rx.numpy().reshape(world * T, H)
        rids = rids.numpy().reshape(world * T, K)
        rw = rw.numpy().reshape(world * T, K)
        # 3. partial sums with the shard, 4. back to the tokens' ranks
        part = partial_sums(haro, lg, lu, ld, El, rx, rids, rw)
        back = torch.empty(world * T * H)
        dist.all_to_all_single(back, torch.from_numpy(part.reshape(-1)))
        back = back.numpy().reshape(world, T, H)
        # 5. shared expert gated by sigmoid(gi . x), residual, partials in rank order
        g = np.array([haro.sigmoid(float(np.dot(gi.astype(np.float64), x[t]))) for t in range(T)],
                     np.float32)
        ysh = haro.moe_ffn(sg, su, sd, None, None, 1, H, I, x, np.zeros((T, 1), np.int32),
                           g.reshape(T, 1))
        y = x + ysh
        for d in range(world):
            y = y + back[d]
        ref = haro.moe_ffn(hg, hu, hd, (sg, su, sd), gi, E, H, I, x, ids, w, add_residual=True)
        err = float(np.abs(y - ref).max() / np.abs(ref).max())
        assert rb == H // 256 * 144
        assert err < 1e-5, err
        # the plan sends each (token, expert) pair to exactly one rank
        assert int((lids >= 0).sum()) == T * K
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok", err))
    except Exception as e:  # report to the parent instead of hanging it
        import traceback
        q.put((rank, "fail", traceback.format_exc() + str(e)))


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_ep_dataflow_matches_unsharded_layer():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = []
    try:
        for _ in procs:
            results.append(q.get(timeout=300))
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    for rank, status, info in results:
        assert status == "ok", f"rank {rank}: {info}"
