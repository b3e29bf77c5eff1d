"""har_cuda_moe_ffn_noalloc against har_cuda_moe_ffn, through the C ABI.

The no-allocation entry point serves callers that cannot call cudaMalloc
(runtimes that reserve the GPU's memory up front for their own pools, hot
loops that cannot take an allocation's synchronisation).  It runs the same
kernels on a static device scratch array instead of the context's arena, so
its results must match the regular entry point within the parity tolerance,
call after call, even though every call reuses the array the previous call
left behind.  This file is collected last so that a `-x` run has executed
every other test before it; it also passes alone in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

import haro  # noqa: E402
import har_cuda  # noqa: E402
from _common import assert_close  # noqa: E402
from gpu_util import Layer, to_dev  # noqa: E402

E, H, I, K = 64, 2048, 512, 10


@pytest.fixture(scope="module")
def ctx():
    c = har_cuda.Context(0)
    yield c
    torch.cuda.synchronize()
    c.close()


@pytest.fixture(scope="module")
def layer(ctx):
    return Layer(ctx, E, H, I, seed=31337)


def call_regular(ctx, lay, x, ids, w, flags):
    xd, idd, wd = to_dev(x), to_dev(ids), to_dev(w)
    y = torch.empty_like(xd)
    ctx.moe_ffn(lay.layer, xd, idd, wd, y, flags)
    ctx.synchronize()
    return y.cpu().numpy()


def call_noalloc(ctx, lay, x, ids, w, flags):
    xd, idd, wd = to_dev(x), to_dev(ids), to_dev(w)
    y = torch.empty_like(xd)
    torch.cuda.synchronize()
    T, k = ids.shape
    st = ctx.lib.har_cuda_moe_ffn_noalloc(ctx.handle, lay.layer.handle, C.c_void_p(xd.data_ptr()),
                                          T, k, C.c_void_p(idd.data_ptr()),
                                          C.c_void_p(wd.data_ptr()), C.c_void_p(y.data_ptr()),
                                          flags)
    ctx.check(st)
    ctx.synchronize()
    return y.cpu().numpy()


@pytest.mark.parametrize("flags", [0, har_cuda.MOE_ACT_Q8K | har_cuda.MOE_ADD_RESIDUAL])
def test_noalloc_matches_moe_ffn_twice(ctx, layer, flags):
    for call in range(2):  # two calls in a row, different inputs each time
        T = 24 + 9 * call
        x = haro.normal_f32(700 + call, 0, T * H).reshape(T, H)
        ids, w = haro.zipf_routing(800 + call, T, E, K)
        ref = call_regular(ctx, layer, x, ids, w, flags)
        got = call_noalloc(ctx, layer, x, ids, w, flags)
        assert_close(got, ref, what=f"noalloc call {call}")


def test_noalloc_second_call_allocates_nothing(ctx, layer):
    T = 16
    x = haro.normal_f32(900, 0, T * H).reshape(T, H)
    ids, w = haro.zipf_routing(901, T, E, K)
    xd, idd, wd = to_dev(x), to_dev(ids), to_dev(w)
    y = torch.empty_like(xd)
    ctx.moe_ffn_noalloc(layer.layer, xd, idd, wd, y)   # first call on the device: set-up
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info(0)[0]
    ctx.moe_ffn_noalloc(layer.layer, xd, idd, wd, y)
    ctx.synchronize()
    assert torch.cuda.mem_get_info(0)[0] == free0


def test_noalloc_rejects_calls_beyond_its_scratch(ctx, layer):
    T = 1024  # needs far more than the 32 MiB static scratch
    xd = torch.zeros((T, H), dtype=torch.float32, device="cuda")
    idd = torch.zeros((T, K), dtype=torch.int32, device="cuda")
    wd = torch.zeros((T, K), dtype=torch.float32, device="cuda")
    y = torch.empty_like(xd)
    with pytest.raises(har_cuda.HarCudaError) as e:
        ctx.moe_ffn_noalloc(layer.layer, xd, idd, wd, y)
    assert e.value.status == har_cuda.ERR_GEOMETRY
    assert "static scratch" in str(e.value)
