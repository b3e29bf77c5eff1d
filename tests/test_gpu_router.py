"""Router on the device: the f32 router GEMV (routed_moe's
self.matvec(ffn_gate_inp), har/crates/har-demo/src/bin/har-native-qwen35moe.rs:1168-1172
with dot_f32_row :154-163), the whole selection (:1167-1204) and routed_moe
(:1167-1215) through the C ABI, against the CPU restatement.

Logits and expert ids are integer-exact work for this path (the top-k order
depends on every bit of the logits), so they are compared bit for bit; the
weights are bit-exact against the oracle's correctly rounded exp mode (the
GPU router's exp) and within 1e-6 of the glibc-expf mode; the layer output
uses the layer tolerances of the other MoE tests."""
import numpy as np
import pytest

import haro
from _common import TC_NRMS, assert_close


def test_router_logits_oracle_is_sequential_f32():
    """The restatement of dot_f32_row: one f32 accumulator, index order, each
    product rounded before the add (no fused multiply-add)."""
    rng = np.random.default_rng(3)
    E, H = 5, 77
    w = rng.standard_normal((E, H)).astype(np.float32)
    x = rng.standard_normal((2, H)).astype(np.float32)
    got = haro.router_logits(w, x)
    for t in range(2):
        for e in range(E):
            s = np.float32(0.0)
            for h in range(H):
                s = np.float32(s + np.float32(w[e, h] * x[t, h]))
            assert got[t, e] == s


def _router(E, H, seed, dup=None):
    w = haro.normal_f32(seed, 0, E * H, 0.0, 0.02).reshape(E, H)
    if dup is not None:
        for a, b in dup:  # identical rows -> identical logits -> a tie
            w[b] = w[a]
    return np.ascontiguousarray(w)


@pytest.mark.gpu
@pytest.mark.parametrize("T,E,H", [(1, 512, 2048), (37, 100, 333), (256, 512, 2048),
                                   (70, 33, 64), (5, 8, 1),
                                   # decode-sized batches (T <= 16), E not a multiple of 8,
                                   # H not a multiple of the 128-wide slice
                                   (2, 512, 2048), (4, 100, 512), (3, 7, 64),
                                   (8, 512, 2048), (16, 100, 260), (11, 9, 4),
                                   # T > 512: four tokens per thread, a ragged last tile
                                   (600, 64, 256)])
def test_router_logits_bit_exact(T, E, H):
    import torch
    from gpu_util import to_dev
    import har_cuda

    ctx = har_cuda.Context(0)
    w = _router(E, H, 11 + T)
    x = haro.normal_f32(12 + T, 0, T * H).reshape(T, H)
    out = torch.full((T, E), float("nan"), dtype=torch.float32, device="cuda")
    ctx.router_logits(to_dev(w), to_dev(x), out)
    torch.cuda.synchronize()
    ctx.synchronize()
    ref = haro.router_logits(w, x)
    got = out.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    ctx.close()


@pytest.mark.gpu
@pytest.mark.parametrize("T,E,H,k", [(1, 512, 2048, 10), (64, 512, 2048, 10), (33, 64, 512, 8),
                                     (3, 32, 256, 32), (8, 512, 2048, 10), (16, 100, 260, 8),
                                     (13, 64, 2048, 32)])
def test_route_from_tokens_bit_exact(T, E, H, k):
    import torch
    from gpu_util import to_dev
    import har_cuda

    ctx = har_cuda.Context(0)
    w = _router(E, H, 21 + T, dup=[(3, 9), (0, E - 1)])
    x = haro.normal_f32(22 + T, 0, T * H).reshape(T, H)
    ids = torch.full((T, k), -7, dtype=torch.int32, device="cuda")
    wts = torch.full((T, k), float("nan"), dtype=torch.float32, device="cuda")
    ctx.route(to_dev(w), to_dev(x), k, ids, wts)
    torch.cuda.synchronize()
    ctx.synchronize()
    logits = haro.router_logits(w, x)
    har_ids, har_w = haro.route_topk(logits, k, exp_mode=0)   # glibc expf, as Rust
    gi, gw = ids.cpu().numpy(), wts.cpu().numpy()
    assert np.array_equal(gi, har_ids)
    assert np.array_equal(gw.view(np.uint32), har_w.view(np.uint32))
    ctx.close()


@pytest.mark.gpu
@pytest.mark.parametrize("T,flags", [(3, 0), (40, 0), (5, 0x4)])
def test_routed_moe_matches_oracle(T, flags):
    """routed_moe on the device: the route record bit-exact, the output within
    the layer tolerances (tensor-core default, CUDA-core GEMV with FORCE_GEMV)."""
    import torch
    from gpu_util import Layer, to_dev
    import har_cuda

    ctx = har_cuda.Context(0)
    E, H, I, k = 16, 2048, 512, 4
    L = Layer(ctx, E, H, I, 500)
    w = _router(E, H, 31)
    x = haro.normal_f32(32 + T, 0, T * H).reshape(T, H)
    xd = to_dev(x)
    ids = torch.empty((T, k), dtype=torch.int32, device="cuda")
    wts = torch.empty((T, k), dtype=torch.float32, device="cuda")
    y = torch.empty_like(xd)
    ctx.routed_moe(L.layer, to_dev(w), xd, k, ids, wts, y, flags)
    torch.cuda.synchronize()
    ctx.synchronize()
    ref_ids, ref_w = haro.route_topk(haro.router_logits(w, x), k, exp_mode=0)
    assert np.array_equal(ids.cpu().numpy(), ref_ids)
    assert np.array_equal(wts.cpu().numpy().view(np.uint32), ref_w.view(np.uint32))
    ref = L.oracle(x, ref_ids, ref_w)
    if flags & har_cuda.MOE_FORCE_GEMV:
        assert_close(y.cpu().numpy(), ref, what="routed_moe gemv")
    else:
        assert_close(y.cpu().numpy(), ref, nrms=TC_NRMS, what="routed_moe tc")
    ctx.close()


@pytest.mark.gpu
def test_route_argument_errors():
    import torch
    import har_cuda

    ctx = har_cuda.Context(0)
    E, H = 64, 128
    w = torch.zeros((E, H), dtype=torch.float32, device="cuda")
    x = torch.zeros((2, H), dtype=torch.float32, device="cuda")
    ids = torch.empty((2, 33), dtype=torch.int32, device="cuda")
    wts = torch.empty((2, 33), dtype=torch.float32, device="cuda")
    with pytest.raises(har_cuda.HarCudaError) as e:
        ctx.route(w, x, 33, ids, wts)                     # k > 32
    assert e.value.status == har_cuda.ERR_GEOMETRY
    lib = ctx.lib
    st = lib.har_cuda_router_logits(ctx.handle, None, E, H, x.data_ptr(), 2, x.data_ptr())
    assert st == har_cuda.ERR_ARG
    st = lib.har_cuda_router_logits(ctx.handle, w.data_ptr(), E, 0, x.data_ptr(), 2, x.data_ptr())
    assert st == har_cuda.ERR_GEOMETRY
    # T = 0 is a no-op
    assert lib.har_cuda_route(ctx.handle, w.data_ptr(), E, H, x.data_ptr(), 0, 4,
                              ids.data_ptr(), wts.data_ptr()) == har_cuda.OK
    ctx.close()
