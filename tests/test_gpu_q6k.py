"""Q6_K GEMV: the CPU restatement of q6k_dot
(har/crates/har-demo/src/bin/har-native-qwen3.rs:174-205) checked on
hand-built blocks, and the CUDA kernel (har_cuda_q6k_gemv, through the C ABI)
against it on seeded blocks at odd and full sizes.

The reference holds no Q6_K test vector, so the hand-built blocks below pin the
restatement to the block layout the reference reads (ql / qh / int8 scales /
f16 d); the GPU kernel is floating-point work with its own summation order,
held to the path's bounds: max|d| / max|ref| <= 1e-3 and HAR's differential
verdict (normalised RMS <= 5e-5)."""
import numpy as np
import pytest

import haro
from _common import assert_close

ZERO_QH = 0xAA  # code 32 (value 0) in every 2-bit high field: nibble 0, high bits 0b10


def _block(d=1.0, scales=None):
    b = np.zeros(210, np.uint8)
    b[128:192] = ZERO_QH
    sc = np.ones(16, np.int8) if scales is None else np.asarray(scales, np.int8)
    b[192:208] = sc.view(np.uint8)
    b[208:210] = np.array([d], np.float16).view(np.uint8)
    return b


def _set_code(b, pos, code):
    """Write 6-bit `code` at value position pos = half*128 + g*32 + l."""
    half, g, l = pos // 128, (pos % 128) // 32, pos % 32
    qi = half * 64 + (g % 2) * 32 + l
    q, h = int(b[qi]), int(b[128 + half * 32 + l])
    if g < 2:
        q = (q & 0xF0) | (code & 15)
    else:
        q = (q & 0x0F) | ((code & 15) << 4)
    h = (h & (0xFF ^ (3 << (2 * g)))) | (((code >> 4) & 3) << (2 * g))
    b[qi] = q
    b[128 + half * 32 + l] = h


def test_q6k_all_ones_block_dot_is_256():
    b = _block(1.0)
    b[0:128] = 0x11                  # nibble 1 everywhere
    b[128:192] = 0xAA                # high bits 0b10 -> code 33, value 1
    assert haro.q6k_dot(b, np.ones(256, np.float32)) == 256.0


def test_q6k_value_positions_and_scales():
    """Every position alone: dot with the unit vector = d * scale * (code - 32),
    scale index half*8 + l/16 + 2g."""
    scales = np.arange(-8, 8, dtype=np.int8) * 3 + 1
    d = 0.5
    for pos in range(256):
        half, g, l = pos // 128, (pos % 128) // 32, pos % 32
        code = (pos * 7 + 5) % 64
        b = _block(d, scales)
        _set_code(b, pos, code)
        x = np.zeros(256, np.float32)
        x[pos] = 1.0
        want = np.float32(d) * (np.float32(scales[half * 8 + l // 16 + 2 * g]) *
                                np.float32(code - 32))
        assert haro.q6k_dot(b, x) == want, pos


def test_q6k_zero_block_dot_is_zero():
    b = _block(1.0)
    x = np.random.default_rng(0).standard_normal(256).astype(np.float32)
    assert haro.q6k_dot(b, x) == 0.0


@pytest.mark.gpu
@pytest.mark.parametrize("N,K,M", [(1, 256, 1), (7, 512, 2), (333, 768, 3), (4096, 4096, 1),
                                   (2048, 2048, 5), (64, 5120, 9), (300, 2048, 16),
                                   # batch-1 rows streamed through shared memory (K % 2048 == 0):
                                   # a ragged last stage, a two-stage ring, fewer rows than SMs
                                   (5000, 2048, 1), (150, 6144, 1), (7, 2048, 1)])
def test_q6k_gemv_matches_restatement(N, K, M):
    import torch
    import har_cuda
    from gpu_util import to_dev

    ctx = har_cuda.Context(0)
    E = 2
    wb = haro.random_q6k(40 + N + K, E * N, K)
    w = ctx.upload(har_cuda.GGML_Q6_K, wb, E, N, K)
    x = haro.normal_f32(41 + M, 0, M * K).reshape(M, K)
    y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    for e in range(E):
        ctx.q6k_gemv(w, e, to_dev(x), M, y)
        torch.cuda.synchronize()
        ctx.synchronize()
        ref = haro.q6k_matvec(wb[e * N:(e + 1) * N], N, K, x)
        assert_close(y.cpu().numpy(), ref, what=f"q6k N={N} K={K} M={M} e={e}")
    w.free()
    ctx.close()


@pytest.mark.gpu
def test_q6k_type_checks():
    """Each entry point takes only the block type it computes on."""
    import torch
    import har_cuda

    ctx = har_cuda.Context(0)
    q6 = ctx.upload(har_cuda.GGML_Q6_K, haro.random_q6k(1, 4, 256), 1, 4, 256)
    q4 = ctx.upload_q4k(np.zeros(4 * 144, np.uint8), 1, 4, 256)
    x = torch.zeros((1, 256), dtype=torch.float32, device="cuda")
    y = torch.zeros((1, 4), dtype=torch.float32, device="cuda")
    with pytest.raises(har_cuda.HarCudaError) as e:
        ctx.q6k_gemv(q4, 0, x, 1, y)
    assert e.value.status == har_cuda.ERR_UNSUPPORTED
    with pytest.raises(har_cuda.HarCudaError) as e:
        ctx.q4k_gemv(q6, 0, x, har_cuda.ACT_F32, 1, y)
    assert e.value.status == har_cuda.ERR_UNSUPPORTED
    with pytest.raises(har_cuda.HarCudaError) as e:
        ctx.q6k_gemv(q6, 1, x, 1, y)                 # expert out of range
    assert e.value.status == har_cuda.ERR_ARG
    with pytest.raises(har_cuda.HarCudaError) as e:
        ctx.upload(3, np.zeros(16, np.uint8), 1, 1, 256)   # unsupported type id
    q6.free()
    q4.free()
    ctx.close()
