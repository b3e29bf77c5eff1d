"""GPU parity of the tensor-core (tcgen05) expert path against the oracle's
restatement of compose_moe_route (har-native-qwen35moe.rs:979-1048).

The default tensor-core path computes exact sc*q weights, the min term from
hi/lo splits and the super-block scales in f32 (activations as hi/lo f16
pairs): it meets HAR's differential verdict, normalised RMS <= 5e-5, like the
f32 CUDA-core path.  The opt-in HAR_CUDA_MOE_TC_F16W variant rounds each
weight to f16 and is held to the north star's max|d|/max|ref| <= 1e-3 with an
RMS bound of 6e-4."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

import haro  # noqa: E402
import har_cuda  # noqa: E402
from _common import F16W_NRMS, TC_NRMS, VERDICT_NRMS, assert_close, verdict  # noqa: E402
from gpu_util import Layer  # noqa: E402

FORCE_TC = har_cuda.MOE_FORCE_TC


@pytest.fixture(scope="module")
def ctx():
    c = har_cuda.Context(0)
    yield c
    torch.cuda.synchronize()
    c.close()


@pytest.fixture(scope="module")
def small(ctx):
    # 64 experts of the Alice shape (hidden 2048, intermediate 512) + shared expert
    return Layer(ctx, 64, 2048, 512, seed=4242)


def test_tc_decode_token(ctx, small):
    x = haro.normal_f32(1, 0, 2048).reshape(1, 2048)
    ids, w = haro.route_topk(haro.normal_f32(2, 0, 64).reshape(1, 64), 10)
    y = small.run(ctx, x, ids, w, FORCE_TC)
    assert_close(y, small.oracle(x, ids, w), nrms=TC_NRMS, what="tc T=1")


def test_tc_zipf_batch(ctx, small):
    x = haro.normal_f32(3, 0, 64 * 2048).reshape(64, 2048)
    ids, w = haro.zipf_routing(4, 64, 64, 10)
    ref = small.oracle(x, ids, w)
    assert_close(small.run(ctx, x, ids, w, FORCE_TC), ref, nrms=TC_NRMS, what="tc forced")
    # hot experts on tcgen05, the tail on the CUDA-core GEMV
    ctx.set_tc_min_tokens(8)
    try:
        assert_close(small.run(ctx, x, ids, w), ref, nrms=TC_NRMS, what="mixed")
        # Q8_K activations keep every expert on the GEMV kernels
        assert_close(small.run(ctx, x, ids, w, har_cuda.MOE_ACT_Q8K),
                     small.oracle(x, ids, w, act="q8k"), rel=1e-4, nrms=1e-5, what="q8k")
    finally:
        ctx.set_tc_min_tokens(0)


def test_tc_prefill_tiles(ctx, small):
    # hundreds of tokens on one expert: several 32-token tiles, shared expert on tcgen05
    T = 300
    x = haro.normal_f32(5, 0, T * 2048).reshape(T, 2048)
    ids, w = haro.route_topk(haro.normal_f32(6, 0, T * 64).reshape(T, 64), 10)
    y = small.run(ctx, x, ids, w, har_cuda.MOE_ADD_RESIDUAL)
    assert_close(y, small.oracle(x, ids, w, residual=True), nrms=TC_NRMS, what="prefill")


def test_tc_batched_equals_isolated(ctx, small):
    x = haro.normal_f32(7, 0, 5 * 2048).reshape(5, 2048)
    ids, w = haro.zipf_routing(8, 5, 64, 10)
    yb = small.run(ctx, x, ids, w, FORCE_TC)
    for t in range(5):
        ys = small.run(ctx, x[t:t + 1], ids[t:t + 1], w[t:t + 1], FORCE_TC)
        assert np.array_equal(ys[0], yb[t]), t


def test_tc_other_shapes(ctx):
    # H = 1024, I = 256 (one 128-row tile pair less), no shared expert
    lay = Layer(ctx, 16, 1024, 256, seed=99, shared=False)
    x = haro.normal_f32(9, 0, 40 * 1024).reshape(40, 1024)
    ids, w = haro.zipf_routing(10, 40, 16, 4)
    assert_close(lay.run(ctx, x, ids, w, FORCE_TC), lay.oracle(x, ids, w), nrms=TC_NRMS,
                 what="tc H=1024")


@pytest.mark.parametrize("I", [768, 1024])
def test_tc_down_stage_layouts(ctx, I):
    # the down GEMM's K (= I) at 12 and 16 K-steps per tile, on the 256-row
    # paired tiles, against the oracle
    lay = Layer(ctx, 8, 1024, I, seed=31 + I, shared=True)
    x = haro.normal_f32(12, 0, 24 * 1024).reshape(24, 1024)
    ids, w = haro.zipf_routing(13, 24, 8, 3)
    assert_close(lay.run(ctx, x, ids, w, FORCE_TC), lay.oracle(x, ids, w), nrms=TC_NRMS,
                 what=f"tc I={I}")


def test_tc_f16w_variant(ctx, small):
    # the opt-in f16-weight variant against the oracle, and the default path's
    # margin on the same tokens
    x = haro.normal_f32(41, 0, 64 * 2048).reshape(64, 2048)
    ids, w = haro.zipf_routing(42, 64, 64, 10)
    ref = small.oracle(x, ids, w)
    y16 = small.run(ctx, x, ids, w, FORCE_TC | har_cuda.MOE_TC_F16W)
    assert_close(y16, ref, nrms=F16W_NRMS, what="tc f16w")
    y = small.run(ctx, x, ids, w, FORCE_TC)
    assert_close(y, ref, nrms=VERDICT_NRMS, what="tc exact")
    assert verdict(y, ref)[0] < 0.1 * verdict(y16, ref)[0]
    # f16w decode token and down-stage layouts
    x1 = haro.normal_f32(43, 0, 2048).reshape(1, 2048)
    i1, w1 = haro.route_topk(haro.normal_f32(44, 0, 64).reshape(1, 64), 10)
    assert_close(small.run(ctx, x1, i1, w1, har_cuda.MOE_TC_F16W), small.oracle(x1, i1, w1),
                 nrms=F16W_NRMS, what="tc f16w T=1")


def test_tc_zero_and_offset_blocks(ctx):
    # super-blocks with d = 0 (only the min term) and with d shrunk 1024-fold
    # under an unchanged dmin (dmin >= 512 d: the unit scale's shift e > 0),
    # written by hand into a layer's weights; values stay in f16 range
    lay = Layer(ctx, 4, 1024, 256, seed=77, shared=False)
    for dev_t, host in ((lay.dg, lay.hg), (lay.du, lay.hu), (lay.dd, lay.hd)):
        hb = host.reshape(-1, 144)
        hb[0::3, 0:2] = 0                          # d = 0 in every third block
        d16 = np.frombuffer(hb[1::3, 0:2].tobytes(), np.float16).astype(np.float32)
        hb[1::3, 0:2] = (d16 / 1024.0).astype(np.float16).view(np.uint8).reshape(-1, 2)
        dev_t.copy_(torch.from_numpy(host.reshape(-1)).to(dev_t.device))
    torch.cuda.synchronize()
    x = haro.normal_f32(45, 0, 24 * 1024).reshape(24, 1024)
    ids, w = haro.zipf_routing(46, 24, 4, 2)
    ref = lay.oracle(x, ids, w)
    assert_close(lay.run(ctx, x, ids, w, FORCE_TC), ref, nrms=TC_NRMS, what="tc d=0 / small d")
    assert_close(lay.run(ctx, x, ids, w, har_cuda.MOE_FORCE_GEMV), ref, what="gemv d=0 / small d")


def test_tc_reports_values_beyond_f16(ctx, small):
    # activations travel as f16 hi/lo pairs on the tensor-core path: a token
    # with |x| >= 65520 sets the device error word instead of returning
    # silent infinities; the CUDA-core path takes it
    x = haro.normal_f32(47, 0, 3 * 2048).reshape(3, 2048)
    x[1, 5] = 1.0e5
    ids, w = haro.route_topk(haro.normal_f32(48, 0, 3 * 64).reshape(3, 64), 10)
    with pytest.raises(har_cuda.HarCudaError) as e:
        small.run(ctx, x, ids, w, FORCE_TC)
    assert e.value.status == har_cuda.ERR_DEVICE
    ctx.synchronize()
    y = small.run(ctx, x, ids, w, har_cuda.MOE_FORCE_GEMV)
    assert np.isfinite(y).all()
