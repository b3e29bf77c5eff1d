"""The opt-in decode path (HAR_CUDA_MOE_DECODE) against the oracle's
compose_moe_route (har-native-qwen35moe.rs:979-1048), through the C ABI.

For at most 8 tokens per call the layer runs as two launches without the
expert-major grouping: one for every selected expert's gate/up with SwiGLU
(plus the shared expert's gate), one for every slot's down rows with the
weighted combine and the residual.  f32 activations on CUDA cores: HAR's
differential verdict (normalised RMS <= 5e-5) holds, and a token's result
does not depend on the other tokens of the call."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

import haro  # noqa: E402
import har_cuda  # noqa: E402
from _common import assert_close  # noqa: E402
from gpu_util import Layer, to_dev  # noqa: E402

E, H, I, K = 64, 2048, 512, 10
DEC = har_cuda.MOE_DECODE


@pytest.fixture(scope="module")
def ctx():
    c = har_cuda.Context(0)
    yield c
    torch.cuda.synchronize()
    c.close()


@pytest.fixture(scope="module")
def layer(ctx):
    return Layer(ctx, E, H, I, seed=7100)


def routing(T, seed):
    return haro.route_topk(haro.normal_f32(seed, 0, T * E).reshape(T, E), K)


@pytest.mark.parametrize("T,flags", [(1, 0), (3, har_cuda.MOE_ADD_RESIDUAL), (8, 0)])
def test_decode_matches_oracle(ctx, layer, T, flags):
    x = haro.normal_f32(7101 + T, 0, T * H).reshape(T, H)
    ids, w = routing(T, 7111 + T)
    y = layer.run(ctx, x, ids, w, DEC | flags)
    ref = layer.oracle(x, ids, w, residual=bool(flags & har_cuda.MOE_ADD_RESIDUAL))
    assert_close(y, ref, what=f"decode T={T}")


def test_decode_batched_equals_isolated(ctx, layer):
    T = 6
    x = haro.normal_f32(7121, 0, T * H).reshape(T, H)
    ids, w = routing(T, 7122)
    yb = layer.run(ctx, x, ids, w, DEC)
    for t in range(T):
        ys = layer.run(ctx, x[t:t + 1], ids[t:t + 1], w[t:t + 1], DEC)
        assert np.array_equal(ys[0], yb[t]), t


def test_decode_layer_without_shared_expert(ctx):
    lay = Layer(ctx, 16, 1024, 256, seed=7130, shared=False)
    x = haro.normal_f32(7131, 0, 2 * 1024).reshape(2, 1024)
    ids, w = haro.route_topk(haro.normal_f32(7132, 0, 2 * 16).reshape(2, 16), 4)
    assert_close(lay.run(ctx, x, ids, w, DEC), lay.oracle(x, ids, w), what="decode no shared")


def test_routed_decode_matches_oracle(ctx, layer):
    T, k = 2, K
    router = haro.normal_f32(7141, 0, E * H, 0.0, 0.02).reshape(E, H)
    x = haro.normal_f32(7142, 0, T * H).reshape(T, H)
    xd = to_dev(x)
    ids = torch.empty((T, k), dtype=torch.int32, device="cuda")
    wts = torch.empty((T, k), dtype=torch.float32, device="cuda")
    y = torch.empty_like(xd)
    ctx.routed_moe(layer.layer, to_dev(router), xd, k, ids, wts, y, DEC)
    torch.cuda.synchronize()
    ctx.synchronize()
    ref_ids, ref_w = haro.route_topk(haro.router_logits(router, x), k, exp_mode=0)
    assert np.array_equal(ids.cpu().numpy(), ref_ids)
    assert np.array_equal(wts.cpu().numpy().view(np.uint32), ref_w.view(np.uint32))
    assert_close(y.cpu().numpy(), layer.oracle(x, ref_ids, ref_w), what="routed decode")


def test_decode_argument_errors(ctx, layer):
    x = np.zeros((9, H), np.float32)
    ids, w = routing(9, 7151)
    with pytest.raises(har_cuda.HarCudaError) as e:
        layer.run(ctx, x, ids, w, DEC)                      # more than 8 tokens
    assert e.value.status == har_cuda.ERR_GEOMETRY
    with pytest.raises(har_cuda.HarCudaError) as e:
        layer.run(ctx, x[:1], ids[:1], w[:1], DEC | har_cuda.MOE_ACT_Q8K)
    assert e.value.status == har_cuda.ERR_ARG
    bad = ids[:1].copy()
    bad[0, 3] = E + 2                                      # out-of-range id: device error word
    with pytest.raises(har_cuda.HarCudaError):
        layer.run(ctx, x[:1], bad, w[:1], DEC)
    ctx.synchronize()
