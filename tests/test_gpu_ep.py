"""Expert parallelism on two GPUs of one box (har_cuda_ep_moe_ffn / _stack).

Each rank holds half of the routed experts and the shared expert; its tokens
go to the experts' ranks and their partial sums come back, through the NCCL
rounds (the default) or peer memory (windows mapped by CUDA IPC, rows pulled
over NVLink).  Per rank, the result must equal the unsharded layer run on
that GPU alone (har_cuda_moe_ffn / _moe_stack) up to f32 summation order, and
the two transports must agree exactly (the same rows reach the same expert
launches; the peer path only leaves out the zero partial sums).  Runs as two
child processes, one per GPU; skipped with fewer than two GPUs.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
mp = pytest.importorskip("torch.multiprocessing")

import har_cuda  # noqa: E402

E, H, I, K, T = 16, 1024, 512, 4, 24
RB_H, RB_I = H // 256 * 144, I // 256 * 144


def gen(ctx, dev, rows, k_dim, seed):
    t = torch.empty(rows * (k_dim // 256) * 144, dtype=torch.uint8, device=dev)
    ctx.gen_q4k(t, rows, k_dim, seed)
    return t


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
        ep = ctx.ep_create(box[0], world, rank)
        lo, hi = har_cuda.expert_range(E, world, rank)
        El = hi - lo
        layers, locals_, shareds, gates = [], [], [], []
        keep = []
        for l in range(2):
            s0 = 700 + 10 * l
            dg, du, dd = gen(ctx, dev, E * I, H, s0 + 1), gen(ctx, dev, E * I, H, s0 + 2), gen(ctx, dev, E * H, I, s0 + 3)
            sg, su, sd = gen(ctx, dev, I, H, s0 + 4), gen(ctx, dev, I, H, s0 + 5), gen(ctx, dev, H, I, s0 + 6)
            gi = torch.from_numpy(haro.normal_f32(s0 + 7, 0, H, 0.0, 0.02)).to(dev)
            keep += [dg, du, dd, sg, su, sd, gi]
            full = ctx.moe_layer(ctx.wrap_q4k(dg, E, I, H), ctx.wrap_q4k(du, E, I, H),
                                 ctx.wrap_q4k(dd, E, H, I),
                                 (ctx.wrap_q4k(sg, 1, I, H), ctx.wrap_q4k(su, 1, I, H),
                                  ctx.wrap_q4k(sd, 1, H, I)), gi)
            local = ctx.moe_layer(ctx.wrap_q4k(dg[lo * I * RB_H:hi * I * RB_H], El, I, H),
                                  ctx.wrap_q4k(du[lo * I * RB_H:hi * I * RB_H], El, I, H),
                                  ctx.wrap_q4k(dd[lo * H * RB_I:hi * H * RB_I], El, H, I))
            shared = ctx.moe_layer(ctx.wrap_q4k(sg, 1, I, H), ctx.wrap_q4k(su, 1, I, H),
                                   ctx.wrap_q4k(sd, 1, H, I))
            layers.append(full)
            locals_.append(local)
            shareds.append(shared)
            gates.append(gi)
        x = torch.from_numpy(haro.normal_f32(40 + rank, 0, T * H).reshape(T, H)).to(dev)
        idw = [haro.zipf_routing(50 + 7 * l + rank, T, E, K) for l in range(2)]
        ids = torch.from_numpy(np.stack([a for a, _ in idw])).to(dev)
        w = torch.from_numpy(np.stack([b for _, b in idw])).to(dev)
        errs = []
        for flags in (har_cuda.MOE_ADD_RESIDUAL, har_cuda.MOE_ADD_RESIDUAL | har_cuda.MOE_ACT_Q8K,
                      har_cuda.MOE_ADD_RESIDUAL | har_cuda.MOE_FORCE_GEMV):
            for call in range(2):  # twice in a row: exchange buffers are reused
                y_ep = torch.empty_like(x)
                ctx.ep_moe_ffn(ep, locals_[0], shareds[0], gates[0], x, ids[0], w[0], y_ep, flags)
                y_ref = torch.empty_like(x)
                ctx.moe_ffn(layers[0], x, ids[0], w[0], y_ref, flags)
                torch.cuda.synchronize()
                ctx.synchronize()
                a, b = y_ep.cpu().numpy(), y_ref.cpu().numpy()
                err = float(np.abs(a - b).max() / np.abs(b).max())
                errs.append(err)
                assert err < 1e-5, (flags, call, err)
            ys = torch.empty_like(x)
            ctx.ep_moe_stack(ep, locals_, shareds, gates, x, ids, w, ys, flags)
            yr = torch.empty_like(x)
            ctx.moe_stack(layers, x, ids, w, yr, flags)
            torch.cuda.synchronize()
            ctx.synchronize()
            a, b = ys.cpu().numpy(), yr.cpu().numpy()
            err = float(np.abs(a - b).max() / np.abs(b).max())
            errs.append(err)
            assert err < 1e-5, (flags, "stack", err)
        assert ep.exchange_mode == 0
        # the two transports on the same stack, both twice (windows and flags reused)
        outs = {}
        for p2p in (False, True, False, True):
            ep.set_p2p(p2p)
            yo = torch.empty_like(x)
            ctx.ep_moe_stack(ep, locals_, shareds, gates, x, ids, w, yo, har_cuda.MOE_ADD_RESIDUAL)
            torch.cuda.synchronize()
            ctx.synchronize()
            outs.setdefault(p2p, []).append(yo.cpu().numpy())
        mode = ep.exchange_mode
        assert mode in (1, -1), mode  # peer memory, or NCCL where the windows cannot be mapped
        for p2p, ys_ in outs.items():
            assert np.array_equal(ys_[0], ys_[1]), ("repeat", p2p)
        assert np.array_equal(outs[False][0], outs[True][0]), "peer memory and NCCL differ"
        dist.barrier()
        ep.free()
        dist.destroy_process_group()
        q.put((rank, "ok", (max(errs), mode)))
    except Exception as e:  # report to the parent instead of hanging it
        import traceback
        q.put((rank, "fail", traceback.format_exc() + str(e)))


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_ep_two_gpus_match_single_gpu_layer():
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
            results.append(q.get(timeout=600))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank, status, info in results:
        assert status == "ok", f"rank {rank}: {info}"
