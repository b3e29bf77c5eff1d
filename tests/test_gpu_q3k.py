"""Q3_K GEMV: the CUDA kernel (har_cuda_q3k_gemv, through the C ABI) against
the oracle's Q3_K restatement on seeded blocks at odd and full sizes.

The reference records Q3_K's geometry only (har/crates/har-model/src/lib.rs:591)
and holds no Q3_K arithmetic or vectors: the oracle restates the GGUF block
layout (pinned to hand-built blocks in tests/test_oracle_q3k.py), so parity
here is unpinned against the reference.  The kernel is floating-point work
with its own summation order, held to the path's bounds: max|d| / max|ref|
<= 1e-3 and normalised RMS <= 5e-5."""
import numpy as np
import pytest

import haro
from _common import assert_close


@pytest.mark.gpu
@pytest.mark.parametrize("N,K,M", [(1, 256, 1), (7, 512, 2), (333, 768, 3), (4096, 2048, 1),
                                   (2048, 2048, 5), (64, 5120, 9), (300, 2048, 16),
                                   (5000, 1024, 1)])
def test_q3k_gemv_matches_restatement(N, K, M):
    import torch
    import har_cuda
    from gpu_util import to_dev

    ctx = har_cuda.Context(0)
    E = 2
    wb = haro.random_q3k(60 + N + K, E * N, K)
    w = ctx.upload(har_cuda.GGML_Q3_K, wb, E, N, K)
    x = haro.normal_f32(61 + M, 0, M * K).reshape(M, K)
    y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    for e in range(E):
        ctx.q3k_gemv(w, e, to_dev(x), M, y)
        torch.cuda.synchronize()
        ctx.synchronize()
        ref = haro.q3k_matvec(wb[e * N:(e + 1) * N], N, K, x)
        assert_close(y.cpu().numpy(), ref, what=f"q3k N={N} K={K} M={M} e={e}")
    w.free()
    ctx.close()


@pytest.mark.gpu
def test_q3k_type_checks():
    """The Q3_K GEMV takes only Q3_K weights, and the Q4_K GEMV refuses them."""
    import torch
    import har_cuda

    ctx = har_cuda.Context(0)
    q3 = ctx.upload(har_cuda.GGML_Q3_K, haro.random_q3k(1, 4, 256), 1, 4, 256)
    q4 = ctx.upload_q4k(np.zeros(4 * 144, np.uint8), 1, 4, 256)
    x = torch.zeros((1, 256), dtype=torch.float32, device="cuda")
    y = torch.zeros((1, 4), dtype=torch.float32, device="cuda")
    with pytest.raises(har_cuda.HarCudaError) as e:
        ctx.q3k_gemv(q4, 0, x, 1, y)
    assert e.value.status == har_cuda.ERR_UNSUPPORTED
    with pytest.raises(har_cuda.HarCudaError) as e:
        ctx.q4k_gemv(q3, 0, x, har_cuda.ACT_F32, 1, y)
    assert e.value.status == har_cuda.ERR_UNSUPPORTED
    with pytest.raises(har_cuda.HarCudaError) as e:
        ctx.q3k_gemv(q3, 1, x, 1, y)                 # expert out of range
    assert e.value.status == har_cuda.ERR_ARG
    q3.free()
    q4.free()
    ctx.close()
