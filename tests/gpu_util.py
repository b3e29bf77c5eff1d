"""Helpers for the GPU parity tests: a context, device-generated Q4_K layers
with host copies for the oracle."""
import numpy as np
import torch

import har_cuda

QK = 256
Q4 = 144


def dev():
    return torch.device("cuda", 0)


def to_dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.to(dev())


def gen_tensor(ctx, rows, K, seed):
    """rows x K Q4_K generated on the device; returns (device tensor, host bytes)."""
    t = torch.empty(rows * (K // QK) * Q4, dtype=torch.uint8, device=dev())
    ctx.gen_q4k(t, rows, K, seed)
    torch.cuda.synchronize()
    return t, t.cpu().numpy().reshape(rows, (K // QK) * Q4)


class Layer:
    """A MoE layer (E experts + optional shared expert and gate row)."""

    def __init__(self, ctx, E, H, I, seed, shared=True, gate_row=True):
        self.E, self.H, self.I = E, H, I
        self.dg, self.hg = gen_tensor(ctx, E * I, H, seed + 1)
        self.du, self.hu = gen_tensor(ctx, E * I, H, seed + 2)
        self.dd, self.hd = gen_tensor(ctx, E * H, I, seed + 3)
        wg = ctx.wrap_q4k(self.dg, E, I, H)
        wu = ctx.wrap_q4k(self.du, E, I, H)
        wd = ctx.wrap_q4k(self.dd, E, H, I)
        self.shared_host = None
        sh = None
        self.gi_host = None
        gi_dev = None
        if shared:
            self.dsg, hsg = gen_tensor(ctx, I, H, seed + 4)
            self.dsu, hsu = gen_tensor(ctx, I, H, seed + 5)
            self.dsd, hsd = gen_tensor(ctx, H, I, seed + 6)
            self.shared_host = (hsg, hsu, hsd)
            sh = (ctx.wrap_q4k(self.dsg, 1, I, H), ctx.wrap_q4k(self.dsu, 1, I, H),
                  ctx.wrap_q4k(self.dsd, 1, H, I))
            if gate_row:
                import haro
                self.gi_host = haro.normal_f32(seed + 7, 0, H, 0.0, 0.02)
                gi_dev = to_dev(self.gi_host)
        self.weights = (wg, wu, wd, sh)
        self.gi_dev = gi_dev
        self.layer = ctx.moe_layer(wg, wu, wd, sh, gi_dev)

    def oracle(self, x, ids, w, act="f32", residual=False, threads=0):
        import haro
        return haro.moe_ffn(self.hg, self.hu, self.hd, self.shared_host, self.gi_host, self.E,
                            self.H, self.I, x, ids, w, add_residual=residual, threads=threads,
                            act=act)

    def run(self, ctx, x, ids, w, flags=0):
        xd, idd, wd = to_dev(x), to_dev(ids), to_dev(w)
        y = torch.empty_like(xd)
        ctx.moe_ffn(self.layer, xd, idd, wd, y, flags)
        torch.cuda.synchronize()
        ctx.synchronize()
        return y.cpu().numpy()
