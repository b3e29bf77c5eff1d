#!/usr/bin/env python
"""bench.py — Q4_K MoE-FFN tokens/s and weight GB/s vs HBM peak on B200.

Default workload ("config 5"): the 48-layer
Alice-shaped MoE FFN stack, attention omitted — per layer 512 experts (top-10)
+ one shared expert with a sigmoid gate row, hidden 2048, intermediate 512,
all Q4_K from N(0,0.02); 256 tokens with Zipf(1.1) routing drawn independently
per layer; residual add between layers (y = x + moe(x), as execute_layer_cpu).
A step is one pass of the 256 tokens through all 48 layers.  With N GPUs
(torchrun) each rank has its own 256 tokens and holds 512/N experts of every
layer (expert parallelism: token rows go to the experts' GPUs and partial sums
come back over NCCL, or pulled over NVLink from the ranks' IPC-mapped windows
with --ep-p2p); the job's tokens grow with N ("scaling": "weak").

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--config 1..5] [--act f32|q8k]

One JSON line on rank 0.  `value` is the device-timed throughput with inputs
resident in HBM (CUDA graph replay, CUDA events, max over ranks); `e2e` is the
same metric through the C ABI's host-buffer entry point (host<->device copies
inside the timed region).  `--impl reference` times the reference's CPU path
(the oracle's C restatement, all host threads) on a bounded sample.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "remora-lab_b200"))

E, H, I, TOPK = 512, 2048, 512, 10
EXPERT_BYTES = (2 * I * (H // 256) + H * (I // 256)) * 144  # gate + up + down = 1,769,472 B
METRIC = "Q4_K MoE-FFN tokens/s (+ weight GB/s vs HBM peak)"

CONFIGS = {
    1: dict(name="config1: single Q4_K GEMV 4096x4096, batch 1", layers=1, T=1),
    2: dict(name="config2: one Alice-shaped MoE layer, decode batch 1, uniform top-10", layers=1, T=1),
    3: dict(name="config3: one MoE layer, 64 concurrent tokens, Zipf(1.1) top-10", layers=1, T=64),
    4: dict(name="config4: one MoE layer, prefill 4096 tokens, uniform top-10", layers=1, T=4096),
    5: dict(name="config5: 48-layer Alice-shaped MoE FFN stack, 256 tokens, Zipf(1.1) top-10",
            layers=48, T=256),
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, choices=sorted(CONFIGS), default=5)
    ap.add_argument("--act", choices=["f32", "q8k"], default="f32",
                    help="activation semantics: f32 (the reference's compose_moe_route; every "
                         "expert on tcgen05) or q8k (Q8_K integer dots on the GEMV kernels)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="target CPU time of the cpu_baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--tc-f16w", action="store_true",
                    help="run the opt-in f16-weight tensor-core variant (HAR_CUDA_MOE_TC_F16W) "
                         "as the timed path")
    ap.add_argument("--ep-p2p", action="store_true",
                    help="with N > 1: move the expert-parallel rows through peer memory (CUDA IPC "
                         "windows over NVLink) instead of NCCL send/recv")
    ap.add_argument("--profile-only", action="store_true",
                    help="run warm-up + a few steps only (for ncu launch lists)")
    ap.add_argument("--routed-decode", action="store_true",
                    help="one JSON line for serving-style decode: the 48-layer stack with every "
                         "layer routed on the device (har_cuda_routed_moe_stack) at T = 1, 8, 64; "
                         "not the driver's bench line")
    ap.add_argument("--rd-batches", default="1,8,64",
                    help="--routed-decode: comma-separated tokens per step")
    ap.add_argument("--rd-paths", default="default,tc_f16w,gemv,decode",
                    help="--routed-decode: comma-separated paths to time")
    ap.add_argument("--layers", type=int, default=None,
                    help="override the layer count (small ncu captures only; the bench "
                         "line always uses the config's 48)")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# synthetic inputs (seeded; the oracle consumes the same bytes in cpu_baseline)
# ---------------------------------------------------------------------------

def zipf_routing(seed: int, T: int, n_exp: int, k: int, s: float = 1.1):
    """Zipf(s) top-k distinct expert ids per token; ranks mapped through a seeded
    permutation (hot experts spread over expert-parallel shards); weights are
    a softmax over seeded N(0,1) logits of the k selected."""
    rng = np.random.default_rng(seed)
    p = np.arange(1, n_exp + 1, dtype=np.float64) ** (-s)
    p /= p.sum()
    perm = rng.permutation(n_exp).astype(np.int32)
    ids = np.empty((T, k), np.int32)
    for t in range(T):
        got = []
        while len(got) < k:
            draw = rng.choice(n_exp, size=2 * k, p=p)
            for d in draw:
                e = int(perm[d])
                if e not in got:
                    got.append(e)
                    if len(got) == k:
                        break
        ids[t] = got
    lg = rng.standard_normal((T, k))
    w = np.exp(lg - lg.max(axis=1, keepdims=True))
    w = (w / w.sum(axis=1, keepdims=True)).astype(np.float32)
    return ids, w


def uniform_routing(seed: int, T: int, n_exp: int, k: int):
    """Top-k of a softmax over seeded N(0,1) logits (distinct, uniform over experts);
    weights renormalised over the selected, as routed_moe computes them."""
    rng = np.random.default_rng(seed)
    lg = rng.standard_normal((T, n_exp)).astype(np.float32)
    ids = np.argsort(-lg, axis=1, kind="stable")[:, :k].astype(np.int32)
    sel = np.take_along_axis(lg, ids, axis=1).astype(np.float64)
    w = np.exp(sel - sel.max(axis=1, keepdims=True))
    return ids, (w / w.sum(axis=1, keepdims=True)).astype(np.float32)


# ---------------------------------------------------------------------------
# clocks sampler (nvidia-smi during the timed region)
# ---------------------------------------------------------------------------

class Clocks:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.device)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# the stack on the device
# ---------------------------------------------------------------------------

def build_stack(ctx, torch, cfg_id: int, rank: int, n_layers=None):
    """Weights generated on the device (the library's generator), routing and
    activations on the host with numpy."""
    dev = torch.device("cuda", ctx.device)
    cfg = CONFIGS[cfg_id]
    L, T = n_layers or cfg["layers"], cfg["T"]
    layers, keep, dist = [], [], []
    import har_cuda  # noqa: F401
    for l in range(L):
        seed = 1000 + 17 * l
        t = {}
        for name, rows, K in (("gate", E * I, H), ("up", E * I, H), ("down", E * H, I),
                              ("sg", I, H), ("su", I, H), ("sd", H, I)):
            buf = torch.empty(rows * (K // 256) * 144, dtype=torch.uint8, device=dev)
            ctx.gen_q4k(buf, rows, K, seed + len(t))
            t[name] = buf
        gi = torch.from_numpy(np.random.default_rng(seed).standard_normal(H).astype(np.float32)
                              * np.float32(0.02)).to(dev)
        wg = ctx.wrap_q4k(t["gate"], E, I, H)
        wu = ctx.wrap_q4k(t["up"], E, I, H)
        wd = ctx.wrap_q4k(t["down"], E, H, I)
        sh = (ctx.wrap_q4k(t["sg"], 1, I, H), ctx.wrap_q4k(t["su"], 1, I, H),
              ctx.wrap_q4k(t["sd"], 1, H, I))
        layers.append(ctx.moe_layer(wg, wu, wd, sh, gi))
        keep.append((t, gi))
    rng = np.random.default_rng(77 + rank)
    x = rng.standard_normal((T, H)).astype(np.float32)
    ids = np.empty((L, T, TOPK), np.int32)
    w = np.empty((L, T, TOPK), np.float32)
    for l in range(L):
        if cfg_id in (3, 5):
            ids[l], w[l] = zipf_routing(500 + 31 * l + 1000 * rank, T, E, TOPK)
        else:
            ids[l], w[l] = uniform_routing(500 + 31 * l + 1000 * rank, T, E, TOPK)
        dist.append(len(np.unique(ids[l])))
    torch.cuda.synchronize()
    return layers, keep, x, ids, w, dist


def routing(cfg_id: int, rank: int, L: int, T: int):
    """The per-layer routing of `rank`'s T tokens ([L][T][k] ids and weights)."""
    ids = np.empty((L, T, TOPK), np.int32)
    w = np.empty((L, T, TOPK), np.float32)
    for l in range(L):
        gen = zipf_routing if cfg_id in (3, 5) else uniform_routing
        ids[l], w[l] = gen(500 + 31 * l + 1000 * rank, T, E, TOPK)
    return ids, w


def build_ep_stack(ctx, torch, cfg_id: int, rank: int, world: int):
    """Rank `rank`'s share of the stack for expert parallelism: its routed
    experts [lo, hi) of every layer (the same bytes as the unsharded stack:
    the generator is seeded per tensor and indexed by row), the shared expert
    as a one-expert layer, and the gate row; its own T tokens and routing.
    distinct[l] counts the experts of layer l that any rank's tokens reach
    (the weights read per layer over the whole job, shared experts apart)."""
    import har_cuda
    dev = torch.device("cuda", ctx.device)
    cfg = CONFIGS[cfg_id]
    L, T = cfg["layers"], cfg["T"]
    lo, hi = har_cuda.expert_range(E, world, rank)
    El = hi - lo
    locals_, shareds, gates, keep = [], [], [], []
    for l in range(L):
        seed = 1000 + 17 * l
        t = {}
        for j, (name, rows, K, row0) in enumerate((
                ("gate", El * I, H, lo * I), ("up", El * I, H, lo * I), ("down", El * H, I, lo * H),
                ("sg", I, H, 0), ("su", I, H, 0), ("sd", H, I, 0))):
            buf = torch.empty(rows * (K // 256) * 144, dtype=torch.uint8, device=dev)
            ctx.gen_q4k(buf, rows, K, seed + j, row0)
            t[name] = buf
        gi = torch.from_numpy(np.random.default_rng(seed).standard_normal(H).astype(np.float32)
                              * np.float32(0.02)).to(dev)
        locals_.append(ctx.moe_layer(ctx.wrap_q4k(t["gate"], El, I, H),
                                     ctx.wrap_q4k(t["up"], El, I, H),
                                     ctx.wrap_q4k(t["down"], El, H, I)))
        shareds.append(ctx.moe_layer(ctx.wrap_q4k(t["sg"], 1, I, H), ctx.wrap_q4k(t["su"], 1, I, H),
                                     ctx.wrap_q4k(t["sd"], 1, H, I)))
        gates.append(gi)
        keep.append((t, gi))
    x = np.random.default_rng(77 + rank).standard_normal((T, H)).astype(np.float32)
    ids, w = routing(cfg_id, rank, L, T)
    all_ids = [routing(cfg_id, r, L, T)[0] for r in range(world)]
    distinct = [len(np.unique(np.concatenate([a[l].ravel() for a in all_ids]))) for l in range(L)]
    local_distinct = [int(np.sum((np.unique(np.concatenate([a[l].ravel() for a in all_ids])) >= lo)
                                 & (np.unique(np.concatenate([a[l].ravel() for a in all_ids])) < hi)))
                      for l in range(L)]
    torch.cuda.synchronize()
    return locals_, shareds, gates, keep, x, ids, w, distinct, local_distinct


def cpu_sample(torch, keep, x, ids, w, seconds: float):
    """The reference's CPU path (oracle restatement of compose_moe_route with
    expert_matvec's per-call row-chunk threads over all host cores) on the
    same weights, routing and tokens, one token at a time, layer after layer,
    for about `seconds` of host time (weight copies to the host not timed).
    Returns (token-layers per second, token-layers done, seconds, layers, cores)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import haro
    cores = haro.online_cpus()
    done, dt, nl = 0, 0.0, 0
    for layer in range(len(keep)):
        t, gi = keep[layer]
        rb = lambda name, rows, K: t[name].cpu().numpy().reshape(rows, K // 256 * 144)  # noqa: E731
        hg, hu, hd = rb("gate", E * I, H), rb("up", E * I, H), rb("down", E * H, I)
        sh = (rb("sg", I, H), rb("su", I, H), rb("sd", H, I))
        gih = gi.cpu().numpy()
        nl += 1
        for n in range(x.shape[0]):
            t0 = time.perf_counter()
            haro.moe_ffn(hg, hu, hd, sh, gih, E, H, I, x[n:n + 1], ids[layer, n:n + 1],
                         w[layer, n:n + 1], add_residual=True, threads=0)
            dt += time.perf_counter() - t0
            done += 1
            if dt >= seconds:
                return done / dt, done, dt, nl, cores
    return done / dt, done, dt, nl, cores


def run_ours(args, torch):
    import har_cuda

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    ctx = har_cuda.Context(local, use_torch_stream=False)
    cfg = CONFIGS[args.config]
    if args.config not in (4, 5):
        raise SystemExit("bench.py times config 5 (default) and config 4 (--config 4); configs "
                         "2-3 are parity-test cases (tests/test_gpu_*.py), config 1 has --config 1")
    if args.layers and not args.profile_only:
        raise SystemExit("--layers is only for --profile-only captures")
    ep = None
    if world > 1:
        # expert parallelism: this rank's expert shard; rows exchanged through
        # NCCL (or peer memory with --ep-p2p)
        locals_, shareds, gates, keep, x, ids, w, distinct, local_distinct = build_ep_stack(
            ctx, torch, args.config, rank, world)
        box = [har_cuda.ep_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        ep = ctx.ep_create(box[0], world, rank, timeout_ms=60000)
        if args.ep_p2p:
            ep.set_p2p(True)
        L = len(locals_)
    else:
        layers, keep, x, ids, w, distinct = build_stack(ctx, torch, args.config, rank, args.layers)
        local_distinct = distinct
        L = len(layers)
    T = cfg["T"]
    flags = har_cuda.MOE_ADD_RESIDUAL | (har_cuda.MOE_ACT_Q8K if args.act == "q8k" else 0) | \
        (har_cuda.MOE_TC_F16W if args.tc_f16w else 0)
    dev = torch.device("cuda", local)
    xd = torch.from_numpy(x).to(dev)
    idd = torch.from_numpy(ids).to(dev)
    wd = torch.from_numpy(w).to(dev)
    yd = torch.empty_like(xd)
    stream = torch.cuda.Stream(dev)
    ctx.lib.har_cuda_ctx_set_stream(ctx.handle, __import__("ctypes").c_void_p(stream.cuda_stream))

    def step(xin, idin, win, yout):
        if ep is not None:
            ctx.ep_moe_stack(ep, locals_, shareds, gates, xin, idin, win, yout, flags)
        else:
            ctx.moe_stack(layers, xin, idin, win, yout, flags)

    # The norm-free stack (BASELINE's "attention omitted": y = x + moe(x) per
    # layer) grows like |x|^2 per layer, so from N(0,1) inputs its activations
    # leave f16 range after about a dozen layers (and f32 range soon after, in
    # the reference's arithmetic as here).  The tensor-core path reports that
    # through the device error word; the work per step does not depend on the
    # values, so the run records the report and goes on.  Per-layer parity at
    # this shape is tested on RMS-normalised inputs (tests/test_gpu_configs.py).
    range_flagged = [False]

    def sync_range():
        try:
            ctx.synchronize()
        except har_cuda.HarCudaError as e:
            if e.status != har_cuda.ERR_DEVICE or "f16 range" not in str(e):
                raise
            range_flagged[0] = True

    # eager warm-up (allocates the scratch arena), then capture one step in a graph
    with torch.cuda.stream(stream):
        for _ in range(2):
            step(xd, idd, wd, yd)
    sync_range()
    torch.cuda.synchronize()
    n0 = ctx.launch_count
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        step(xd, idd, wd, yd)
    launches_per_step = ctx.launch_count - n0
    torch.cuda.synchronize()

    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            g.replay()
    torch.cuda.synchronize()
    if args.profile_only:
        with torch.cuda.stream(stream):
            for _ in range(args.steps):
                g.replay()
        torch.cuda.synchronize()
        return None

    clocks = Clocks(local)
    clocks.start()
    time.sleep(0.5)  # let the sampler come up before the timed region
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        ev0.record(stream)
        for _ in range(args.steps):
            g.replay()
        ev1.record(stream)
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / args.steps
    if dist:
        dist.barrier()
    clk = clocks.stop()
    if dist:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())

    # per-kernel durations: one eager step with the library's CUDA-event profiling
    ctx.profile_begin()
    with torch.cuda.stream(stream):
        step(xd, idd, wd, yd)
    prof = ctx.profile_end()
    kern = {}
    for name, t_ms in prof:
        a = kern.setdefault(name, [0, 0.0])
        a[0] += 1
        a[1] += t_ms
    total_k = sum(v[1] for v in kern.values())

    # e2e: host buffers in and out, copies inside the timed region (one GPU:
    # the host-buffer C-ABI call; expert parallel: pinned copies around the
    # public ep_moe_stack call)
    e2e_steps = max(3, min(args.steps, 20))
    if ep is None:
        def e2e_step():
            try:
                ctx.moe_stack_host(layers, x, ids, w, flags)
            except har_cuda.HarCudaError as e:  # the call completed; only the range report
                if e.status != har_cuda.ERR_DEVICE or "f16 range" not in str(e):
                    raise
                range_flagged[0] = True
    else:
        xh = torch.from_numpy(x).pin_memory()
        ih = torch.from_numpy(ids).pin_memory()
        wh = torch.from_numpy(w).pin_memory()
        yh = torch.empty_like(xh).pin_memory()

        def e2e_step():
            with torch.cuda.stream(stream):
                xd.copy_(xh, non_blocking=True)
                idd.copy_(ih, non_blocking=True)
                wd.copy_(wh, non_blocking=True)
                step(xd, idd, wd, yd)
                yh.copy_(yd, non_blocking=True)
            stream.synchronize()
            sync_range()
    for _ in range(2):
        e2e_step()
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    e2e_ms = (time.perf_counter() - t0) * 1e3 / e2e_steps
    if dist:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())

    # the opt-in f16-weight tensor-core variant (HAR_CUDA_MOE_TC_F16W: each
    # dequantised weight rounded to f16, max relative error ~4e-4, not HAR's
    # 5e-5 RMS verdict), timed the same way for comparison
    var = None
    if args.act == "f32" and not args.tc_f16w:
        vflags = flags | har_cuda.MOE_TC_F16W
        with torch.cuda.stream(stream):
            step_v = (lambda: ctx.ep_moe_stack(ep, locals_, shareds, gates, xd, idd, wd, yd, vflags)) \
                if ep is not None else (lambda: ctx.moe_stack(layers, xd, idd, wd, yd, vflags))
            step_v()
        torch.cuda.synchronize()
        gv = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gv, stream=stream):
            step_v()
        with torch.cuda.stream(stream):
            for _ in range(max(3, args.warmup)):
                gv.replay()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        ev0.record(stream)
        with torch.cuda.stream(stream):
            for _ in range(args.steps):
                gv.replay()
        ev1.record(stream)
        torch.cuda.synchronize()
        vms = ev0.elapsed_time(ev1) / args.steps
        if dist:
            t = torch.tensor([vms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            vms = float(t.item())
        ctx.profile_begin()
        with torch.cuda.stream(stream):
            step_v()
        vprof = ctx.profile_end()
        vk = {}
        for name, t_ms in vprof:
            a = vk.setdefault(name, [0, 0.0])
            a[0] += 1
            a[1] += t_ms
        del gv
        var = (vms, vk)

    # algorithmic bytes: each distinct routed expert once per layer over the
    # job, plus the shared expert once per rank; the roofline kernel's bytes are
    # this rank's (its reached local experts and the shared expert)
    step_bytes = sum((d + world) * EXPERT_BYTES for d in distinct)
    gu_bytes = [(d + 1) * 2 * I * (H // 256) * 144 for d in local_distinct]
    peaks = load_peaks()
    hbm = peaks.get("hbm_gbs", 6650.0)
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    # the dominant kernel: the tensor-core gate/up GEMM (every expert takes the
    # tensor-core path at the default threshold); the GEMV kernel otherwise
    rk = next((n for n in ("moe_tc_gate_up_kernel", "moe_tc_f16w_gate_up_kernel") if n in kern),
              "moe_gate_up_kernel")
    gu = kern.get(rk, [1, 1.0])
    # all launches of the kernel in one step: bytes they move / time they take
    achieved = sum(gu_bytes) / (gu[1] * 1e-3) / 1e9
    traffic = load_traffic(rk + ("@config4" if args.config == 4 else ""))
    # config 4 (prefill, ~80 tokens per expert) is bound by the tensor pipe:
    # its roofline is the gate/up kernel's algorithmic FLOPs (2 per multiply-add
    # of the routed and shared experts' gate and up GEMMs) per launch over the
    # measured dense bf16 peak (sustained: the kernel runs inside a long loop)
    tensor_roof = None
    if args.config == 4:
        # per rank: its T tokens' slot rows (T*k over the job spread evenly) and
        # its own T shared-expert rows
        gu_flops = T * (TOPK + 1) * 2 * (2 * H * I)
        tf_sus = peaks.get("bf16_tflops_sustained", 1400.0)
        tf_burst = peaks.get("bf16_tflops", 1590.0)
        ach_tf = gu_flops / (gu[1] * 1e-3) / 1e12
        step_flops = world * T * (TOPK + 1) * 3 * 2 * H * I
        tensor_roof = {
            "bound": "tensor", "kernel": rk, "achieved": round(ach_tf, 1), "peak": tf_sus,
            "unit": "TFLOP/s", "frac": round(ach_tf / tf_sus, 4),
            "peak_source": "measured (bf16_tflops_sustained)" if "bf16_tflops_sustained" in peaks
                           else "fallback",
            "frac_of_burst_peak": round(ach_tf / tf_burst, 4),
            "traffic": traffic,
            "algorithmic_flops_per_step": int(gu_flops), "kernel_ms_per_step": round(gu[1], 4),
            "launches_per_step": gu[0],
            "note": "f16 hi/lo activations double the MMA N: the tensor pipe executes twice "
                    "the algorithmic FLOPs",
            "step_tflops": round(step_flops / world / (ms * 1e-3) / 1e12, 1),
            "step_frac": round(step_flops / world / (ms * 1e-3) / 1e12 / tf_sus, 4)}
    out = None
    if rank == 0:
        tokens_per_s = world * T / (ms * 1e-3)
        out = {
            "metric": METRIC, "value": round(tokens_per_s, 1), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": ("f16 x f16 -> f32 (tcgen05: exact sc*q weights and hi/lo f16 activations, "
                      "super-block scales and mins applied in f32)"
                      if "moe_tc_gate_up_kernel" in kern else
                      "f16 x f16 -> f32 (tcgen05; Q4_K weights rounded to f16 on chip: "
                      "HAR_CUDA_MOE_TC_F16W)" if "moe_tc_f16w_gate_up_kernel" in kern else
                      "int8 x q4 (dp4a) -> i32, f32 combine" if args.act == "q8k" else "f32"),
            "data": "synthetic: N(0,0.02) weights quantised to Q4_K on device; N(0,1) f32 "
                    "activations; " + ("uniform top-10 routing (softmax weights of N(0,1) "
                                       "logits)" if args.config == 4 else
                                       "Zipf(1.1) top-10 routing drawn per layer"),
            "config": {"workload": cfg["name"], "tokens_per_rank": T, "layers": L, "experts": E,
                       "hidden": H, "intermediate": I, "top_k": TOPK, "shared_expert": True,
                       "activations": args.act,
                       "parallelism": f"ep{world}: {E // world} experts per rank" if world > 1
                       else "single",
                       "ep_exchange": None if ep is None else
                       {1: "peer memory (CUDA IPC windows, rows pulled over NVLink)",
                        0: "NCCL send/recv", -1: "NCCL send/recv (windows could not be mapped)"}
                       [ep.exchange_mode],
                       "l2": "inputs larger than L2 (%.1f GB of Q4_K weights read per step)"
                             % (step_bytes / 1e9),
                       "graph": "one CUDA graph per step"},
            "weight_gbs": round(step_bytes / (ms * 1e-3) / 1e9, 1),
            "hbm_frac": round(step_bytes / (ms * 1e-3) / 1e9 / hbm / world, 4),
            "roofline": tensor_roof or {
                "bound": "hbm", "kernel": rk,
                "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(achieved / hbm, 4), "peak_source": peak_src,
                "traffic": traffic,
                "algorithmic_bytes_per_step": int(sum(gu_bytes)),
                "kernel_ms_per_step": round(gu[1], 4), "launches_per_step": gu[0]},
            "kernels": {k: {"launches": v[0], "ms": round(v[1], 4),
                            "share": round(v[1] / total_k, 4)} for k, v in sorted(kern.items())},
            "e2e": {"value": round(world * T / (e2e_ms * 1e-3), 1), "unit": "tokens/s",
                    "ms_per_step": round(e2e_ms, 4),
                    "h2d_bytes_per_step": int(x.nbytes + ids.nbytes + w.nbytes),
                    "d2h_bytes_per_step": int(x.nbytes)},
            "clocks": clk,
            "numerics": {"range_flagged": range_flagged[0],
                         "note": "the norm-free stack's activations leave f16 range after about a "
                                 "dozen layers from N(0,1) inputs (the reference's f32 overflows "
                                 "later); the tensor-core path reports it and the timed work is "
                                 "value-independent; per-layer parity at this shape is tested on "
                                 "RMS-normalised inputs"},
            "variant_tc_f16w": None if var is None else {
                "flag": "HAR_CUDA_MOE_TC_F16W",
                "numerics": "weights rounded to f16: max|d|/max|ref| ~4e-4, nrms ~4e-4 (north "
                            "star's 1e-3; not HAR's 5e-5 verdict, which the default meets)",
                "value": round(world * T / (var[0] * 1e-3), 1), "unit": "tokens/s",
                "ms_per_step": round(var[0], 4),
                "kernels": {k: {"launches": v[0], "ms": round(v[1], 4)} for k, v in sorted(var[1].items())},
                "gate_up_frac_of_hbm": round(sum(gu_bytes) / (var[1].get("moe_tc_f16w_gate_up_kernel",
                                                                          [1, 1e9])[1] * 1e-3) / 1e9 / hbm, 4)},
            "gpu_launches": int(launches_per_step * args.steps),
            "distinct_experts_per_layer": {"min": min(distinct), "max": max(distinct),
                                           "mean": round(sum(distinct) / len(distinct), 1)},
        }
        if world == 1 and not args.no_cpu_baseline:
            tps, n, dt, nl, cores = cpu_sample(torch, keep, x, ids, w, args.cpu_seconds)
            out["cpu_baseline"] = {
                "value": round(tps / L, 3), "unit": "tokens/s", "cores": cores, "kind": "port",
                "sample": f"{n} token-layers of the same stack (layers 0..{nl - 1}, tokens one "
                          f"at a time, {dt:.1f} s of host time): oracle compose_moe_route with "
                          f"expert_matvec row threads over {cores} cores; token-layers/s / {L}"}
    if dist:
        dist.barrier()
        del g  # the graph holds NCCL work: release it before the communicators
        torch.cuda.synchronize()
        if ep is not None:
            ep.free()
        dist.destroy_process_group()
    return out


def run_reference(args):
    """Reference arm: the reference's CPU path for this workload (the oracle's
    C restatement of compose_moe_route; HAR's Rust cannot be built here), all
    host threads, each step a bounded sample of one token through one layer."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import haro
    cfg = CONFIGS[args.config]
    L, T = cfg["layers"], cfg["T"]
    tok = 2  # tokens per step
    ids, w = zipf_routing(500, T, E, TOPK)
    used = sorted(set(ids[:tok].ravel().tolist()))
    remap = {e: i for i, e in enumerate(used)}
    Eu = len(used)
    # weights of the used experts only (the CPU path reads nothing else)
    hg = np.concatenate([haro.gen_q4k(1000, I, H, row0=e * I) for e in used])
    hu = np.concatenate([haro.gen_q4k(1001, I, H, row0=e * I) for e in used])
    hd = np.concatenate([haro.gen_q4k(1002, H, I, row0=e * H) for e in used])
    sh = (haro.gen_q4k(1003, I, H), haro.gen_q4k(1004, I, H), haro.gen_q4k(1005, H, I))
    gi = haro.normal_f32(1006, 0, H, 0.0, 0.02)
    x = np.random.default_rng(77).standard_normal((tok, H)).astype(np.float32)
    lid = np.vectorize(remap.get)(ids[:tok]).astype(np.int32)
    cores = haro.online_cpus()

    def step():
        haro.moe_ffn(hg, hu, hd, sh, gi, Eu, H, I, x, lid, w[:tok], add_residual=True, threads=0)

    for _ in range(max(1, args.warmup)):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    tps = tok / dt / L
    return {
        "impl": "reference", "metric": METRIC, "value": round(tps, 3), "unit": "tokens/s",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: N(0,0.02) Q4_K weights, N(0,1) activations, Zipf(1.1) routing",
        "config": {"workload": cfg["name"], "layers": L, "experts": E, "hidden": H,
                   "intermediate": I, "top_k": TOPK, "shared_expert": True},
        "cpu_baseline": {"value": round(tps, 3), "unit": "tokens/s", "cores": cores,
                         "kind": "port",
                         "sample": f"each step: {tok} tokens through one layer (compose_moe_route, "
                                   f"expert_matvec row threads over {cores} cores); "
                                   f"tokens/s scaled by 1/{L} layers"},
        "e2e": {"value": round(tps, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


GEMV_N, GEMV_K = 131072, 4096  # one decode GEMV of LM-head size: 302 MB of Q4_K (L2 is 126 MB)
GEMV_N_SMALL = 65536            # half the rows, reported beside: the fixed cost per launch shows


def run_gemv_roofline(args, torch):
    """Config 1's kernel, the batch-1 Q4_K GEMV (har_cuda_q4k_gemv), measured as
    a decode roofline: y = W x with W a 131072 x 4096 Q4_K matrix (302 MB, the
    size of an LM-head GEMV) and x one f32 row quantised to Q8_K (config 1's
    activations), alternating between two such matrices so the working set is
    far larger than L2.  The value is weight bytes streamed per second; f32
    activations and the 65536-row matrix are reported beside it.  One JSON
    line; not the driver's bench line (config 5)."""
    import har_cuda

    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    ctx = har_cuda.Context(local, use_torch_stream=False)
    stream = torch.cuda.Stream(dev)
    ctx.lib.har_cuda_ctx_set_stream(ctx.handle, __import__("ctypes").c_void_p(stream.cuda_stream))
    N, K = GEMV_N, GEMV_K
    wbytes = N * (K // 256) * 144
    mats, keep = [], []
    for i in range(2):
        t = torch.empty(wbytes, dtype=torch.uint8, device=dev)
        ctx.gen_q4k(t, N, K, 9100 + i)
        keep.append(t)
        mats.append(ctx.wrap_q4k(t, 1, N, K))
    # the same bytes seen as two matrices of half the rows each
    small = [ctx.wrap_q4k(t, 2, GEMV_N_SMALL, K) for t in keep]
    x = torch.from_numpy(np.random.default_rng(9200).standard_normal((1, K)).astype(np.float32)).to(dev)
    xq = torch.empty((K // 256) * 292, dtype=torch.uint8, device=dev)
    y = torch.empty((1, N), dtype=torch.float32, device=dev)
    per = 8  # GEMVs per graph, alternating matrices
    peaks = load_peaks()
    hbm = peaks.get("hbm_gbs", 6650.0)
    res = {}
    for act, kind, sm in (("q8k", har_cuda.ACT_Q8K, False), ("f32", har_cuda.ACT_F32, False),
                          ("q8k_small", har_cuda.ACT_Q8K, True)):
        with torch.cuda.stream(stream):
            ctx.q8k_quantize(x, xq)
        src = xq if kind == har_cuda.ACT_Q8K else x
        nb = wbytes // 2 if sm else wbytes

        def gemvs():
            for j in range(per):
                if sm:  # four distinct half-size matrices in turn
                    ctx.q4k_gemv(small[j % 2], (j // 2) % 2, src, kind, 1, y)
                else:
                    ctx.q4k_gemv(mats[j % 2], 0, src, kind, 1, y)

        with torch.cuda.stream(stream):
            gemvs()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            gemvs()
        with torch.cuda.stream(stream):
            for _ in range(max(3, args.warmup)):
                g.replay()
        torch.cuda.synchronize()
        clocks = Clocks(local)
        clocks.start()
        time.sleep(0.5)
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for _ in range(args.steps):
                g.replay()
            ev1.record(stream)
        torch.cuda.synchronize()
        clk = clocks.stop()
        ms = ev0.elapsed_time(ev1) / (args.steps * per)
        gbs = nb / (ms * 1e-3) / 1e9
        res[act] = {"ms_per_gemv": round(ms, 5), "weight_gbs": round(gbs, 1), "frac": round(gbs / hbm, 4),
                    "clocks": clk}
    # Q6_K (the GGUF type of LM heads and of some expert tensors): two 65536 x
    # 4096 Q6_K matrices (220 MB each) of random codes and scales, f32
    # activations, alternating as above.
    n6 = GEMV_N_SMALL
    q6bytes = n6 * (K // 256) * 210
    q6 = []
    for i in range(2):
        t = torch.randint(0, 256, (q6bytes,), dtype=torch.uint8, device=dev,
                          generator=torch.Generator(dev).manual_seed(9300 + i))
        t.view(-1, 210)[:, 208:210] = torch.tensor([0x00, 0x1C], dtype=torch.uint8, device=dev)
        keep.append(t)
        q6.append(ctx.wrap(har_cuda.GGML_Q6_K, t, 1, n6, K))
    y6 = torch.empty((1, n6), dtype=torch.float32, device=dev)

    def time_alternating(gemv, mats):
        """ms per GEMV: `per` launches alternating over mats, in a CUDA graph."""
        with torch.cuda.stream(stream):
            for j in range(per):
                gemv(mats[j % 2], 0, x, 1, y6)
        torch.cuda.synchronize()
        gx = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gx, stream=stream):
            for j in range(per):
                gemv(mats[j % 2], 0, x, 1, y6)
        with torch.cuda.stream(stream):
            for _ in range(max(3, args.warmup)):
                gx.replay()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(args.steps):
                gx.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / (args.steps * per)

    ms6 = time_alternating(ctx.q6k_gemv, q6)
    gbs6 = q6bytes / (ms6 * 1e-3) / 1e9
    # Q3_K (the routed gate/up type of the real Alice model): two 65536 x 4096
    # Q3_K matrices (115 MB each) of random bits and scales, d = 2^-8.
    q3bytes = n6 * (K // 256) * 110
    q3 = []
    for i in range(2):
        t = torch.randint(0, 256, (q3bytes,), dtype=torch.uint8, device=dev,
                          generator=torch.Generator(dev).manual_seed(9500 + i))
        t.view(-1, 110)[:, 108:110] = torch.tensor([0x00, 0x1C], dtype=torch.uint8, device=dev)
        keep.append(t)
        q3.append(ctx.wrap(har_cuda.GGML_Q3_K, t, 1, n6, K))
    ms3 = time_alternating(ctx.q3k_gemv, q3)
    gbs3 = q3bytes / (ms3 * 1e-3) / 1e9
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    # The router on the device (har_cuda_router_logits / har_cuda_route) at the
    # Alice shape, E = 512, H = 2048, k = 10: per call, CUDA-graph replays of
    # 20 calls, at the decode and batch sizes it serves.
    router = {}
    E_r, H_r, k_r = 512, 2048, 10
    gr = torch.Generator(dev).manual_seed(9400)
    w_r = torch.randn(E_r, H_r, device=dev, generator=gr) * 0.02
    for T_r in (1, 64, 256, 4096):
        x_r = torch.randn(T_r, H_r, device=dev, generator=gr)
        lg = torch.empty(T_r, E_r, device=dev)
        ids_r = torch.empty(T_r, k_r, dtype=torch.int32, device=dev)
        wt_r = torch.empty(T_r, k_r, device=dev)
        for name, fn in (("logits", lambda: ctx.router_logits(w_r, x_r, lg)),
                         ("route", lambda: ctx.route(w_r, x_r, k_r, ids_r, wt_r))):
            with torch.cuda.stream(stream):
                for _ in range(3):
                    fn()
            torch.cuda.synchronize()
            gg = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gg, stream=stream):
                for _ in range(20):
                    fn()
            with torch.cuda.stream(stream):
                gg.replay()
                ev0.record(stream)
                for _ in range(10):
                    gg.replay()
                ev1.record(stream)
            torch.cuda.synchronize()
            router[f"{name}_T{T_r}_us"] = round(ev0.elapsed_time(ev1) / 200 * 1000, 2)
            del gg
    ctx.synchronize()
    q = res["q8k"]
    return {
        "metric": "Q4_K decode GEMV weight GB/s (batch 1)", "value": q["weight_gbs"], "unit": "GB/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": q["ms_per_gemv"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8 x q4 (dp4a) -> i32, f32 scales", "data": "synthetic: N(0,0.02) weights "
        "quantised to Q4_K on device; one N(0,1) f32 row quantised to Q8_K",
        "config": {"workload": f"config1 kernel as a decode roofline: {N} x {K} Q4_K GEMV, batch 1",
                   "rows": N, "K": K, "batch": 1, "per_graph": per,
                   "l2": "two 302 MB matrices alternate (604 MB working set > 126 MB L2)"},
        "roofline": {"bound": "hbm", "kernel": "q4k_gemv_kernel", "achieved": q["weight_gbs"],
                     "peak": hbm, "unit": "GB/s", "frac": q["frac"],
                     "peak_source": "measured" if "hbm_gbs" in peaks else "fallback",
                     "algorithmic_bytes_per_launch": wbytes},
        "f32_activations": {"weight_gbs": res["f32"]["weight_gbs"], "frac": res["f32"]["frac"],
                            "ms_per_gemv": res["f32"]["ms_per_gemv"]},
        "rows_65536": {"weight_gbs": res["q8k_small"]["weight_gbs"], "frac": res["q8k_small"]["frac"],
                       "ms_per_gemv": res["q8k_small"]["ms_per_gemv"]},
        "router": dict(router, E=E_r, H=H_r, k=k_r),
        "q6k_f32_65536": {"kernel": "q6k_gemv_stream_kernel", "weight_gbs": round(gbs6, 1),
                          "frac": round(gbs6 / hbm, 4), "ms_per_gemv": round(ms6, 5),
                          "rows": n6, "K": K},
        "q3k_f32_65536": {"kernel": "q3k_gemv_smem_kernel", "weight_gbs": round(gbs3, 1),
                          "frac": round(gbs3 / hbm, 4), "ms_per_gemv": round(ms3, 5),
                          "rows": n6, "K": K},
        "clocks": q["clocks"],
    }


def run_routed_decode(args, torch):
    """Serving-style decode over config 5's 48-layer stack: each step routes
    every layer on the device from that layer's input (f32 routers
    N(0, 0.02) [E][H], the reference's routed_moe order) and applies it with the
    residual, all in one har_cuda_routed_moe_stack call captured in a CUDA
    graph; T tokens per step.  Weight GB/s counts each distinct routed expert
    of every layer once (read from the step's route records) plus the shared
    expert."""
    import har_cuda

    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    ctx = har_cuda.Context(local, use_torch_stream=False)
    stream = torch.cuda.Stream(dev)
    ctx.lib.har_cuda_ctx_set_stream(ctx.handle, __import__("ctypes").c_void_p(stream.cuda_stream))
    layers, keep, _, _, _, _ = build_stack(ctx, torch, 5, 0)
    L = len(layers)
    g = torch.Generator(dev).manual_seed(9500)
    routers = [torch.randn(E, H, device=dev, generator=g) * 0.02 for _ in range(L)]
    peaks = load_peaks()
    hbm = peaks.get("hbm_gbs", 6650.0)
    out = {}
    # the default path (every expert on the f32-grade tensor-core kernels), the
    # opt-in f16-weight tensor-core variant and the CUDA-core GEMV path
    # and the decode path (HAR_CUDA_MOE_DECODE, at most 8 tokens per call)
    paths = {"default": 0, "tc_f16w": har_cuda.MOE_TC_F16W, "gemv": har_cuda.MOE_FORCE_GEMV,
             "decode": har_cuda.MOE_DECODE}
    want = set(args.rd_paths.split(","))
    paths = {k: v for k, v in paths.items() if k in want}
    for T in (int(b) for b in args.rd_batches.split(",")):
        x = torch.randn(T, H, device=dev, generator=g)
        y = torch.empty_like(x)
        ids = torch.empty((L, T, TOPK), dtype=torch.int32, device=dev)
        w = torch.empty((L, T, TOPK), dtype=torch.float32, device=dev)
        row = {}
        for pname, pf in paths.items():
            if pf == har_cuda.MOE_DECODE and T > 8:
                continue
            step = lambda: ctx.routed_moe_stack(layers, routers, x, TOPK, ids, w, y,  # noqa: E731
                                                har_cuda.MOE_ADD_RESIDUAL | pf)
            with torch.cuda.stream(stream):
                for _ in range(max(3, args.warmup)):
                    step()
            torch.cuda.synchronize()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=stream):
                step()
            ev0 = torch.cuda.Event(enable_timing=True)
            ev1 = torch.cuda.Event(enable_timing=True)
            n = max(3, min(args.steps, 50))
            with torch.cuda.stream(stream):
                gr.replay()
                ev0.record(stream)
                for _ in range(n):
                    gr.replay()
                ev1.record(stream)
            torch.cuda.synchronize()
            try:  # the norm-free stack leaves f16 range from N(0,1) inputs (see run_ours)
                ctx.synchronize()
            except har_cuda.HarCudaError as e:
                if e.status != har_cuda.ERR_DEVICE or "f16 range" not in str(e):
                    raise
            del gr
            ms = ev0.elapsed_time(ev1) / n
            d = ids.cpu().numpy()
            wbytes = sum((len(np.unique(d[l])) + 1) * EXPERT_BYTES for l in range(L))
            row[pname] = {"ms_per_step": round(ms, 4), "tokens_per_s": round(T / (ms * 1e-3), 1),
                          "weight_gbs": round(wbytes / (ms * 1e-3) / 1e9, 1),
                          "hbm_frac": round(wbytes / (ms * 1e-3) / 1e9 / hbm, 4)}
        out[f"T{T}"] = row
    first_T, first_row = next(iter(out.items()))
    first_path, t1 = next(iter(first_row.items()))
    return {"metric": "routed decode step, 48 Alice-shaped layers, device routing",
            "value": t1["tokens_per_s"], "unit": f"tokens/s ({first_T}, {first_path} path)", "n_gpus": 1,
            "ms_per_step": t1["ms_per_step"], "higher_is_better": True, "dtype": "f32 x, Q4_K W",
            "data": "synthetic: N(0,0.02) Q4_K weights and f32 routers, N(0,1) tokens",
            "config": {"workload": "config 5 stack, har_cuda_routed_moe_stack in one CUDA graph",
                       "layers": L, "experts": E, "k": TOPK, "hidden": H, "inter": I},
            "by_batch": out, "peak_hbm_gbs": hbm}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


def load_traffic(kernel: str):
    """DRAM bytes per launch of `kernel` (key "name" or "name@configN") from the
    committed ncu summaries, if any."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return d.get(kernel, {}).get("traffic_bytes_per_launch")
    except (OSError, ValueError):
        return None


def main():
    args = parse()
    # Only the JSON line goes to stdout: libraries that print at start-up
    # (NCCL's version banner, for one) write to file descriptor 1 directly, so
    # it points at stderr until the result is ready.
    sys.stdout.flush()
    saved = os.dup(1)
    os.dup2(2, 1)
    try:
        if args.impl == "reference":
            out = run_reference(args)
        elif args.routed_decode:
            import torch
            out = run_routed_decode(args, torch)
        elif args.config == 1:
            import torch
            out = run_gemv_roofline(args, torch)
        else:
            import torch
            out = run_ours(args, torch)
    finally:
        sys.stdout.flush()
        os.dup2(saved, 1)
        os.close(saved)
    if out is not None:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
