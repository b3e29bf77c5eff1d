"""GPU parity of the expert-FFN executor (moe_ffn) against the oracle's
restatement of compose_moe_route / routed_moe, through the C ABI."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

import haro  # noqa: E402
import har_cuda  # noqa: E402
from _common import TC_NRMS, assert_close, golden, rel_max  # noqa: E402
from gpu_util import Layer, to_dev  # noqa: E402

E, H, I, K = 512, 2048, 512, 10


@pytest.fixture(scope="module")
def ctx():
    c = har_cuda.Context(0)
    yield c
    torch.cuda.synchronize()
    c.close()


@pytest.fixture(scope="module")
def alice(ctx):
    # One Alice-shaped layer: hidden 2048, 512 experts,
    # intermediate 512, shared expert with a sigmoid gate row, all Q4_K N(0,0.02).
    return Layer(ctx, E, H, I, seed=9000)


def uniform_routing(T, seed):
    logits = haro.normal_f32(seed, 0, T * E).reshape(T, E)
    return haro.route_topk(logits, K)


def test_config2_decode_f32_matches_har(ctx, alice):
    # the f32 CUDA-core GEMV path meets HAR's engine verdict (nrms <= 5e-5)
    x = haro.normal_f32(1, 0, H).reshape(1, H)
    ids, w = uniform_routing(1, 2)
    y = alice.run(ctx, x, ids, w, har_cuda.MOE_FORCE_GEMV)
    assert_close(y, alice.oracle(x, ids, w), what="config2 f32")


def test_config2_decode_default_path(ctx, alice):
    # default: every expert on tcgen05 (f16 weights, hi/lo f16 activations):
    # the north star's max|d|/max|ref| <= 1e-3, RMS within 6e-4
    x = haro.normal_f32(1, 0, H).reshape(1, H)
    ids, w = uniform_routing(1, 2)
    y = alice.run(ctx, x, ids, w)
    assert_close(y, alice.oracle(x, ids, w), nrms=TC_NRMS, what="config2 default")


def test_config2_decode_q8k_matches_q8k_restatement(ctx, alice):
    x = haro.normal_f32(1, 0, H).reshape(1, H)
    ids, w = uniform_routing(1, 2)
    y = alice.run(ctx, x, ids, w, har_cuda.MOE_ACT_Q8K)
    assert_close(y, alice.oracle(x, ids, w, act="q8k"), rel=1e-4, nrms=1e-5, what="config2 q8k")
    assert rel_max(y, alice.oracle(x, ids, w)) < 5e-2


def test_config3_zipf_batch_f32_matches_har(ctx, alice):
    # 64 concurrent tokens, Zipf(1.1) top-10: variable M per expert.  Every
    # expert on the f32 CUDA-core path: HAR's engine verdict (nrms <= 5e-5) holds.
    x = haro.normal_f32(3, 0, 64 * H).reshape(64, H)
    ids, w = haro.zipf_routing(4, 64, E, K)
    y = alice.run(ctx, x, ids, w, har_cuda.MOE_FORCE_GEMV)
    assert_close(y, alice.oracle(x, ids, w), what="config3 f32")


def test_config3_zipf_batch_default_paths(ctx, alice):
    # default threshold: every expert on tcgen05 (max rel 1e-3; RMS 6e-4);
    # then experts with >= 16 tokens on tcgen05 and the tail on the GEMV kernels
    x = haro.normal_f32(3, 0, 64 * H).reshape(64, H)
    ids, w = haro.zipf_routing(4, 64, E, K)
    ref = alice.oracle(x, ids, w)
    assert_close(alice.run(ctx, x, ids, w), ref, nrms=TC_NRMS, what="config3 default")
    ctx.set_tc_min_tokens(16)
    try:
        assert_close(alice.run(ctx, x, ids, w), ref, nrms=TC_NRMS, what="config3 mixed")
    finally:
        ctx.set_tc_min_tokens(0)


def test_config3_zipf_batch_q8k(ctx, alice):
    x = haro.normal_f32(3, 0, 64 * H).reshape(64, H)
    ids, w = haro.zipf_routing(4, 64, E, K)
    y = alice.run(ctx, x, ids, w, har_cuda.MOE_ACT_Q8K | har_cuda.MOE_FORCE_GEMV)
    assert_close(y, alice.oracle(x, ids, w, act="q8k"), rel=1e-4, nrms=1e-5, what="config3 q8k")


@pytest.mark.parametrize("flags", [0, har_cuda.MOE_ACT_Q8K])
def test_batched_equals_isolated(ctx, alice, flags):
    # har/crates/har-serve/src/moe.rs:301-314: bit-exact
    x = haro.normal_f32(5, 0, 5 * H).reshape(5, H)
    ids, w = haro.zipf_routing(6, 5, E, K)
    yb = alice.run(ctx, x, ids, w, flags)
    for t in range(5):
        ys = alice.run(ctx, x[t:t + 1], ids[t:t + 1], w[t:t + 1], flags)
        assert np.array_equal(ys[0], yb[t]), t


def test_residual_and_host_entry_point(ctx, alice):
    x = haro.normal_f32(7, 0, 3 * H).reshape(3, H)
    ids, w = uniform_routing(3, 8)
    yd = alice.run(ctx, x, ids, w, har_cuda.MOE_ADD_RESIDUAL)
    yh = ctx.moe_ffn_host(alice.layer, x, ids, w, har_cuda.MOE_ADD_RESIDUAL)
    assert np.array_equal(yd, yh)
    assert_close(yh, alice.oracle(x, ids, w, residual=True), nrms=TC_NRMS, what="residual")
    yg = ctx.moe_ffn_host(alice.layer, x, ids, w, har_cuda.MOE_ADD_RESIDUAL | har_cuda.MOE_FORCE_GEMV)
    assert_close(yg, alice.oracle(x, ids, w, residual=True), what="residual gemv")


def test_reference_entry_points(ctx, alice):
    m = har_cuda.CudaMoeModel(ctx, [alice.layer], E, H, I, K)
    x = haro.normal_f32(11, 0, H)
    logits = haro.normal_f32(12, 0, E)
    out, ids, w = m.routed_moe(0, x, logits)
    ref_ids, ref_w = haro.route_topk(logits.reshape(1, -1), K)
    assert np.array_equal(ids, ref_ids[0])
    assert rel_max(w, ref_w[0]) < 1e-6
    assert_close(out, alice.oracle(x.reshape(1, -1), ids.reshape(1, -1), w.reshape(1, -1))[0],
                 nrms=TC_NRMS, what="routed_moe")
    g = m.expert_matvec(alice.weights[0], 17, x)
    ref = haro.expert_matvec(alice.hg, E, I, H, 17, x)
    assert_close(g, ref, what="expert_matvec")


def test_layer_without_shared_expert(ctx):
    lay = Layer(ctx, 16, 512, 256, seed=77, shared=False)
    x = haro.normal_f32(1, 0, 9 * 512).reshape(9, 512)
    ids, w = haro.zipf_routing(2, 9, 16, 4)
    ref = lay.oracle(x, ids, w)
    assert_close(lay.run(ctx, x, ids, w), ref, nrms=TC_NRMS, what="no shared")
    assert_close(lay.run(ctx, x, ids, w, har_cuda.MOE_FORCE_GEMV), ref, what="no shared gemv")


def test_shared_expert_without_gate_row(ctx):
    lay = Layer(ctx, 16, 1024, 512, seed=78, shared=True, gate_row=False)
    x = haro.normal_f32(1, 0, 4 * 1024).reshape(4, 1024)
    ids, w = haro.zipf_routing(3, 4, 16, 3)
    ref = lay.oracle(x, ids, w)
    assert_close(lay.run(ctx, x, ids, w), ref, nrms=TC_NRMS, what="shared, no gate")
    assert_close(lay.run(ctx, x, ids, w, har_cuda.MOE_FORCE_GEMV), ref, what="shared, no gate gemv")


def test_golden_moe_fixture(ctx):
    G = golden()
    e, h, i, t, k = (int(v) for v in G["moe_dims"])
    mk = lambda name, n_, k_, ne: ctx.wrap_q4k(to_dev(G[name].reshape(-1)), ne, n_, k_)  # noqa: E731
    keep = [to_dev(G[n].reshape(-1)) for n in ("moe_wg", "moe_wu", "moe_wd", "moe_sg", "moe_su", "moe_sd")]
    wg = ctx.wrap_q4k(keep[0], e, i, h)
    wu = ctx.wrap_q4k(keep[1], e, i, h)
    wd = ctx.wrap_q4k(keep[2], e, h, i)
    sh = (ctx.wrap_q4k(keep[3], 1, i, h), ctx.wrap_q4k(keep[4], 1, i, h), ctx.wrap_q4k(keep[5], 1, h, i))
    gi = to_dev(G["moe_gi"])
    layer = ctx.moe_layer(wg, wu, wd, sh, gi)
    y = ctx.moe_ffn_host(layer, G["moe_x"], G["moe_ids"], G["moe_w"])
    assert_close(y, G["moe_y"], nrms=TC_NRMS, what="golden moe")
    y = ctx.moe_ffn_host(layer, G["moe_x"], G["moe_ids"], G["moe_w"], har_cuda.MOE_FORCE_GEMV)
    assert_close(y, G["moe_y"], what="golden moe gemv")
    del mk


def test_two_layer_stack(ctx, alice):
    lay2 = Layer(ctx, 64, H, I, seed=555)
    # reuse alice as layer 0 only through its first 64 experts' ids
    x = haro.normal_f32(21, 0, 8 * H).reshape(8, H)
    ids0, w0 = haro.zipf_routing(22, 8, 64, K)
    ids1, w1 = haro.zipf_routing(23, 8, 64, K)
    xd = to_dev(x)
    y = torch.empty_like(xd)
    ctx.moe_stack([alice.layer, lay2.layer], xd, to_dev(np.stack([ids0, ids1])),
                  to_dev(np.stack([w0, w1])), y, har_cuda.MOE_ADD_RESIDUAL)
    torch.cuda.synchronize()
    h1 = alice.oracle(x, ids0, w0, residual=True)
    h2 = lay2.oracle(h1, ids1, w1, residual=True)
    assert_close(y.cpu().numpy(), h2, nrms=TC_NRMS, what="stack")


def test_stack_host_repeated_calls(ctx, alice):
    # har_cuda_moe_stack_host replays a CUDA graph from the second call with the
    # same layers and shapes on: every call (new inputs, same shapes; then a
    # changed key) equals the device-buffer stack bit for bit.
    lay2 = Layer(ctx, 64, H, I, seed=556)
    layers = [alice.layer, lay2.layer]

    def device_stack(x, ids, w, flags):
        y = torch.empty((x.shape[0], H), dtype=torch.float32, device=to_dev(x).device)
        ctx.moe_stack(layers, to_dev(x), to_dev(ids), to_dev(w), y, flags)
        torch.cuda.synchronize()
        return y.cpu().numpy()

    f = har_cuda.MOE_ADD_RESIDUAL
    # graph capture needs a real stream (not the legacy default one)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        ctx.bind_torch_stream()
        try:
            for call in range(4):
                x = haro.normal_f32(60 + call, 0, 8 * H).reshape(8, H)
                rw = [haro.zipf_routing(70 + 2 * call + l, 8, 64, K) for l in range(2)]
                ids = np.stack([a for a, _ in rw])
                w = np.stack([b for _, b in rw])
                flags = f if call < 3 else f | har_cuda.MOE_FORCE_GEMV
                yh = ctx.moe_stack_host(layers, x, ids, w, flags)
                assert np.array_equal(yh, device_stack(x, ids, w, flags)), call
        finally:
            torch.cuda.synchronize()
    ctx.bind_torch_stream()


def test_moe_argument_errors(ctx, alice):
    x = np.zeros((1, H), np.float32)
    with pytest.raises(har_cuda.HarCudaError):
        ctx.moe_ffn_host(alice.layer, x, np.zeros((1, E + 1), np.int32), np.zeros((1, E + 1), np.float32))
    with pytest.raises(har_cuda.HarCudaError):
        ctx.moe_ffn_host(alice.layer, x, np.zeros((1, 2), np.int32), np.zeros((1, 2), np.float32),
                         har_cuda.MOE_FORCE_GEMV | har_cuda.MOE_FORCE_TC)
    ids = np.array([[0, E + 5]], np.int32)  # out-of-range expert id: device error word
    with pytest.raises(har_cuda.HarCudaError):
        ctx.moe_ffn_host(alice.layer, x, ids, np.ones((1, 2), np.float32))
    ctx.synchronize()
