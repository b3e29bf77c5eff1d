"""GPU parity of the individual kernels against the oracle, through the C ABI."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

import haro  # noqa: E402
import har_cuda  # noqa: E402
from _common import assert_close, kats, rel_max  # noqa: E402
from gpu_util import dev, gen_tensor, to_dev  # noqa: E402


@pytest.fixture(scope="module")
def ctx():
    c = har_cuda.Context(0)
    yield c
    torch.cuda.synchronize()
    c.close()


def q8k_dev(ctx, x):
    M, K = x.shape
    xd = to_dev(x)
    out = torch.empty((M, K // 256 * 292), dtype=torch.uint8, device=dev())
    ctx.q8k_quantize(xd, out)
    torch.cuda.synchronize()
    return out


def gemv(ctx, w_dev, N, K, x, act):
    M = x.shape[0]
    w = ctx.wrap_q4k(w_dev, 1, N, K)
    y = torch.empty((M, N), dtype=torch.float32, device=dev())
    if act == har_cuda.ACT_Q8K:
        ctx.q4k_gemv(w, 0, q8k_dev(ctx, x), act, M, y)
    else:
        ctx.q4k_gemv(w, 0, to_dev(x), act, M, y)
    torch.cuda.synchronize()
    ctx.synchronize()
    return y.cpu().numpy()


def test_q8k_quantize_bit_exact(ctx):
    x = haro.normal_f32(101, 0, 37 * 2048).reshape(37, 2048)
    x[3, :256] = 0.0                       # all-zero block
    x[4, 256:512] = 1e-40                  # subnormal block
    x[5, 512:768] *= 1e30                  # huge values
    x[6, 1000] = -50.0                     # negative max magnitude
    x[7, :] = np.float32(1.0)              # exact ties at 127
    got = q8k_dev(ctx, x).cpu().numpy()
    assert np.array_equal(got, haro.q8k_quantize(x))


def test_vulkan_smoke_known_answer_on_gpu(ctx):
    # har/crates/har-vulkan/src/bin/smoke.rs:96-160 -> 256.0 within 1e-4
    block = np.zeros(144, np.uint8)
    block[1] = 0x3C
    block[4:16] = 1
    block[16:] = 0x11
    wd = to_dev(block)
    x = np.ones((1, 256), np.float32)
    for act in (har_cuda.ACT_F32, har_cuda.ACT_Q8K):
        y = gemv(ctx, wd, 1, 256, x, act)
        assert abs(float(y[0, 0]) - kats()["vulkan_smoke_q4k_gemv"]["expected"]) < 1e-4


def test_config1_gemv_f32_matches_har_serving_path(ctx):
    # W 4096x4096 N(0,0.02) Q4_K, x N(0,1); HAR's Q4KModel::matvec
    wd, wh = gen_tensor(ctx, 4096, 4096, 1)
    x = haro.normal_f32(2, 0, 4096).reshape(1, 4096)
    y = gemv(ctx, wd, 4096, 4096, x, har_cuda.ACT_F32)
    ref = haro.q4k_matvec(wh, 4096, 4096, x[0])
    assert_close(y[0], ref, what="config1 f32")


def test_config1_gemv_q8k_matches_q8k_restatement(ctx):
    wd, wh = gen_tensor(ctx, 4096, 4096, 1)
    x = haro.normal_f32(2, 0, 4096).reshape(1, 4096)
    y = gemv(ctx, wd, 4096, 4096, x, har_cuda.ACT_Q8K)
    ref = haro.q4k_gemv_q8k(wh, 4096, 4096, haro.q8k_quantize(x))
    assert_close(y[0], ref, rel=1e-5, nrms=1e-6, what="config1 q8k")
    # against HAR's f32-activation path the Q8_K rounding of x dominates
    har = haro.q4k_matvec(wh, 4096, 4096, x[0])
    assert rel_max(y[0], har) < 3e-2


@pytest.mark.parametrize("K", [256, 512, 768, 1024, 2048, 3072, 4096, 5120])
@pytest.mark.parametrize("act", [har_cuda.ACT_F32, har_cuda.ACT_Q8K])
def test_gemv_shapes(ctx, K, act):
    for N, M in ((1, 1), (7, 3), (333, 5), (64, 9)):
        wd, wh = gen_tensor(ctx, N, K, 1000 + K + N)
        x = haro.normal_f32(7 + M, 0, M * K).reshape(M, K)
        y = gemv(ctx, wd, N, K, x, act)
        if act == har_cuda.ACT_F32:
            ref = np.stack([[haro.dot_quant_row(wh[r], x[m]) for r in range(N)] for m in range(M)])
            assert_close(y, ref, what=f"f32 K={K} N={N} M={M}")
        else:
            xq = haro.q8k_quantize(x)
            ref = np.stack([haro.q4k_gemv_q8k(wh, N, K, xq[m]) for m in range(M)])
            assert_close(y, ref, rel=1e-5, nrms=1e-6, what=f"q8k K={K} N={N} M={M}")


@pytest.mark.parametrize("act", [har_cuda.ACT_F32, har_cuda.ACT_Q8K])
def test_model_batched_matches_single(ctx, act):
    # har/crates/har-serve/src/q4k.rs:260-269 and moe.rs:301-314: a batched
    # step equals the sequences run one at a time, bit for bit.
    wd, _ = gen_tensor(ctx, 512, 2048, 77)
    x = haro.normal_f32(78, 0, 6 * 2048).reshape(6, 2048)
    yb = gemv(ctx, wd, 512, 2048, x, act)
    for m in range(6):
        ys = gemv(ctx, wd, 512, 2048, x[m:m + 1], act)
        assert np.array_equal(ys[0], yb[m]), m


def test_cuda_q4k_model_batch_step(ctx):
    # the serving seam over the GPU: BatchStepModel::batch_step semantics
    wd, wh = gen_tensor(ctx, 256, 256, 5)
    embed = haro.lcg_values(256 * 256, 99)
    model = har_cuda.CudaQ4KModel(ctx, wh, 256, 256, embed, eos=7)
    h = model.initial_hidden()
    out = model.batch_step([(h, 1), (h, 2)])
    for (nxt, logits), t in zip(out, (1, 2)):
        xr = h + embed.reshape(256, 256)[t]
        assert np.array_equal(nxt, xr)
        assert np.max(np.abs(logits - haro.q4k_matvec(wh, 256, 256, xr))) < 1e-4  # smoke tolerance
    assert model.weight_bytes_per_row() == 256 * 144


def route(ctx, logits, k):
    T, E = logits.shape
    ld = to_dev(logits)
    ids = torch.empty((T, k), dtype=torch.int32, device=dev())
    w = torch.empty((T, k), dtype=torch.float32, device=dev())
    ctx.route_topk(ld, k, ids, w)
    torch.cuda.synchronize()
    return ids.cpu().numpy(), w.cpu().numpy()


@pytest.mark.parametrize("T,E,k", [(100, 512, 10), (33, 64, 8), (5, 3, 3), (7, 1000, 32)])
def test_route_topk_bit_exact(ctx, T, E, k):
    logits = haro.normal_f32(500 + E, 0, T * E).reshape(T, E)
    ids, w = route(ctx, logits, k)
    # glibc's expf, as Rust's f32::exp: ids and weights bit-exact
    har_ids, har_w = haro.route_topk(logits, k, exp_mode=0)
    assert np.array_equal(ids, har_ids)
    assert np.array_equal(w.view(np.uint32), har_w.view(np.uint32))
    assert np.all(np.abs(w.sum(1) - 1) < 1e-5)


def test_route_topk_ties(ctx):
    logits = np.zeros((4, 16), np.float32)
    logits[1, [3, 9]] = 2.0
    ids, w = route(ctx, logits, 4)
    ref_ids, ref_w = haro.route_topk(logits, 4, exp_mode=0)
    assert np.array_equal(ids, ref_ids) and np.array_equal(w, ref_w)
    assert list(ids[0]) == [0, 1, 2, 3]
    assert list(ids[1][:2]) == [3, 9]


def group(ctx, ids, E):
    T, k = ids.shape
    idd = to_dev(ids)
    counts = torch.empty(E, dtype=torch.int32, device=dev())
    offsets = torch.empty(E + 1, dtype=torch.int32, device=dev())
    order = torch.empty(T * k, dtype=torch.int32, device=dev())
    ctx.group_by_expert(idd, E, counts, offsets, order)
    torch.cuda.synchronize()
    return counts.cpu().numpy(), offsets.cpu().numpy(), order.cpu().numpy()


@pytest.mark.parametrize("T,E,k", [(256, 512, 10), (4096, 512, 10), (1, 512, 10), (3, 2048, 1), (1000, 8, 8),
                                   # above 8192 entries the sort runs over several CTAs:
                                   # a ragged last segment, the largest E, many segments
                                   (2049, 64, 10), (1700, 2048, 10), (40000, 16, 2)])
def test_group_by_expert_bit_exact(ctx, T, E, k):
    ids, _ = haro.zipf_routing(T + E, T, E, k)
    got = group(ctx, ids, E)
    ref = haro.group_by_expert(ids, E)
    for g, r in zip(got, ref):
        assert np.array_equal(g, r)


def test_group_rejects_out_of_range_ids(ctx):
    ids = np.array([[1, 2], [3, 99]], np.int32)
    group(ctx, ids, 8)
    with pytest.raises(har_cuda.HarCudaError) as e:
        ctx.synchronize()
    assert e.value.status == har_cuda.ERR_DEVICE
    ctx.synchronize()  # the error word is cleared after it is reported


def test_group_rejects_out_of_range_ids_across_ctas(ctx):
    ids, _ = haro.zipf_routing(77, 2000, 64, 10)
    ids[1500, 3] = 64
    group(ctx, ids, 64)
    with pytest.raises(har_cuda.HarCudaError) as e:
        ctx.synchronize()
    assert e.value.status == har_cuda.ERR_DEVICE
    ctx.synchronize()


def test_device_generator_matches_host_generator(ctx):
    _, wh = gen_tensor(ctx, 64, 2048, 4242)
    ref = haro.gen_q4k(4242, 64, 2048)
    blocks_equal = np.all(wh.reshape(-1, 144) == ref.reshape(-1, 144), axis=1)
    assert blocks_equal.mean() > 0.99


def test_gemv_argument_errors(ctx):
    wd, _ = gen_tensor(ctx, 8, 256, 3)
    w = ctx.wrap_q4k(wd, 1, 8, 256)
    y = torch.empty((1, 8), dtype=torch.float32, device=dev())
    x = torch.zeros((1, 256), dtype=torch.float32, device=dev())
    with pytest.raises(har_cuda.HarCudaError) as e:
        ctx.q4k_gemv(w, 1, x, har_cuda.ACT_F32, 1, y)   # expert out of range
    assert e.value.status == har_cuda.ERR_ARG
    with pytest.raises(har_cuda.HarCudaError):
        ctx.q4k_gemv(w, 0, x, 7, 1, y)                  # unknown activation kind
    with pytest.raises(har_cuda.HarCudaError) as e:
        ctx.wrap_q4k(wd, 1, 8, 300)                      # K not a multiple of 256
    assert e.value.status == har_cuda.ERR_GEOMETRY


@pytest.mark.parametrize("K", [512, 4096])
@pytest.mark.parametrize("act", [har_cuda.ACT_F32, har_cuda.ACT_Q8K])
def test_gemv_decode_stream(ctx, K, act):
    # batch 1 streams the weights through a shared-memory ring; 12,000 rows give
    # each CTA more stages than ring slots.  Equals the oracle, and equals bit for
    # bit the register-resident kernel's row for the same token (M = 2 call).
    N = 12000
    wd, wh = gen_tensor(ctx, N, K, 4242 + K)
    x = haro.normal_f32(31, 0, 2 * K).reshape(2, K)
    y1 = gemv(ctx, wd, N, K, x[:1], act)
    y2 = gemv(ctx, wd, N, K, x, act)
    assert np.array_equal(y1[0], y2[0])
    if act == har_cuda.ACT_F32:
        assert_close(y1[0], haro.q4k_matvec(wh, N, K, x[0]), what=f"stream f32 K={K}")
    else:
        ref = haro.q4k_gemv_q8k(wh, N, K, haro.q8k_quantize(x[:1])[0])
        assert_close(y1[0], ref, rel=1e-5, nrms=1e-6, what=f"stream q8k K={K}")
