"""GPU parity of the tensor-core (tcgen05) expert path against the oracle's
restatement of compose_moe_route (har-native-qwen35moe.rs:979-1048).

Each dequantised weight is rounded once to f16 on this path (activations go
in as hi/lo f16 pairs, accumulation is f32), so besides the north star's
max|d|/max|ref| <= 1e-3 the RMS bound is 6e-4 instead of the 5e-5 that the
f32 CUDA-core path meets."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

import haro  # noqa: E402
import har_cuda  # noqa: E402
from _common import TC_NRMS, assert_close  # noqa: E402
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
