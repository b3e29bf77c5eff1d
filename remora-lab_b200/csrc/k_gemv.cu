// k_gemv.cu — Q4_K GEMV on CUDA cores for batch-1 and small-M decode:
// y[m][n] = sum_k W_e[n][k] * x[m][k].  Replaces Q4KModel::matvec
// (har/crates/har-serve/src/q4k.rs:170-188), expert_matvec
// (har/crates/har-demo/src/bin/har-native-qwen35moe.rs:626-689) and the
// q4k_gemv / q4k_batched_gemv shaders' role (har/shaders/q4k_gemv.comp,
// har/shaders/q4k_batched_gemv.comp): the same arithmetic, laid out for B200 —
// 128-bit weight loads, activations resident in registers across rows,
// warp-shuffle reduction, MT tokens per weight read.
#include "gemv_engine.cuh"

namespace har {

template <int ACT, int LPR, int CPL, int MT>
__global__ void __launch_bounds__(256) q4k_gemv_kernel(const uint8_t *__restrict__ W, int64_t N,
                                                       int K, int64_t row_bytes,
                                                       const uint8_t *__restrict__ act,
                                                       int64_t act_row_bytes, int M,
                                                       float *__restrict__ y, int rows_per_cta) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ const uint8_t *rowp[MT];
  constexpr int RPW = 32 / LPR;
  const int t0 = blockIdx.y * MT;
  if (threadIdx.x < MT)
    rowp[threadIdx.x] = (t0 + (int)threadIdx.x < M) ? act + (int64_t)(t0 + threadIdx.x) * act_row_bytes : nullptr;
  __syncthreads();
  if (ACT == ACT_F32)
    stage_f32(smem, reinterpret_cast<const float *const *>(rowp), MT, K);
  else
    stage_q8k(smem, rowp, MT, K);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = lane / LPR, gl = lane % LPR;
  const int C = K / 64;
  LaneAct<ACT> a[MT][CPL];
#pragma unroll
  for (int t = 0; t < MT; ++t)
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      const int ch = gl + LPR * i;
      if (ch < C) a[t][i].load(smem, MT, K, t, ch);
    }

  const int64_t r_begin = (int64_t)blockIdx.x * rows_per_cta;
  const int64_t r_end = min(N, r_begin + rows_per_cta);
  for (int64_t rb = r_begin + warp * RPW; rb < r_end; rb += 8 * RPW) {  // warp-uniform
    const int64_t r = rb + grp;
    const bool valid = r < r_end;
    const uint8_t *row = W + (valid ? r : rb) * row_bytes;
    float acc[MT];
#pragma unroll
    for (int t = 0; t < MT; ++t) acc[t] = 0.0f;
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      const int ch = gl + LPR * i;
      if (ch < C) {
        const WChunk w = load_wchunk(row, ch);
#pragma unroll
        for (int t = 0; t < MT; ++t) acc[t] += chunk_dot(w, ch, a[t][i]);
      }
    }
#pragma unroll
    for (int t = 0; t < MT; ++t) acc[t] = lane_group_sum<LPR>(acc[t]);
    if (valid && gl == 0) {
#pragma unroll
      for (int t = 0; t < MT; ++t)
        if (t0 + t < M) y[(int64_t)(t0 + t) * N + r] = acc[t];
    }
  }
}

template <int ACT, int LPR, int CPL, int MT>
static int32_t gemv_launch(har_cuda_ctx *ctx, const uint8_t *W, int64_t N, int K,
                           int64_t row_bytes, const uint8_t *act, int64_t act_row_bytes, int M,
                           float *y) {
  auto kern = q4k_gemv_kernel<ACT, LPR, CPL, MT>;
  const size_t smem = ActSmem<ACT>::bytes(MT, K);
  if (smem > 48 * 1024) {
    if (smem > 200 * 1024) return set_error(ctx, HAR_CUDA_ERR_UNSUPPORTED, "q4k_gemv: K too large");
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  }
  constexpr int RPW = 32 / LPR;
  const int64_t mtiles = (M + MT - 1) / MT;
  // About 4 CTAs per SM in total, each a multiple of one warp pass (8 warps * RPW rows).
  int64_t want = (int64_t)ctx->num_sms * 4 / mtiles;
  if (want < 1) want = 1;
  int64_t rows_per_cta = (N + want - 1) / want;
  rows_per_cta = ((rows_per_cta + 8 * RPW - 1) / (8 * RPW)) * (8 * RPW);
  const int64_t ntiles = (N + rows_per_cta - 1) / rows_per_cta;
  dim3 grid((unsigned)ntiles, (unsigned)mtiles);
  prof_begin(ctx);
  kern<<<grid, 256, smem, ctx->stream>>>(W, N, K, row_bytes, act, act_row_bytes, M, y,
                                         (int)rows_per_cta);
  return check_launch(ctx, "q4k_gemv_kernel");
}

int32_t launch_gemv(har_cuda_ctx *ctx, const har_cuda_weights *w, int64_t expert,
                    const void *x, int act_kind, int64_t M, float *y) {
  const int K = (int)w->K;
  const GemvShape s = gemv_shape(K);
  const uint8_t *W = w->dev + expert * w->expert_bytes;
  const uint8_t *act = (const uint8_t *)x;
  if (act_kind == ACT_F32) {
    if ((uintptr_t)x & 15u) return set_error(ctx, HAR_CUDA_ERR_ARG, "q4k_gemv: x must be 16-byte aligned");
    const int64_t arb = (int64_t)K * 4;
#define F32_CASE(LPR_, CPL_) \
  if (s.LPR == LPR_ && s.CPL == CPL_) return gemv_launch<ACT_F32, LPR_, CPL_, 1>(ctx, W, w->N, K, w->row_bytes, act, arb, (int)M, y);
    F32_CASE(4, 1) F32_CASE(8, 1) F32_CASE(16, 1) F32_CASE(32, 1) F32_CASE(32, 2)
    F32_CASE(32, 3) F32_CASE(32, 4)
#undef F32_CASE
  } else {
    if ((uintptr_t)x & 3u) return set_error(ctx, HAR_CUDA_ERR_ARG, "q4k_gemv: Q8_K rows must be 4-byte aligned");
    const int64_t arb = (int64_t)(K / QK) * Q8K_BYTES;
#define Q8_CASE(LPR_, CPL_, MT_) \
  if (s.LPR == LPR_ && s.CPL == CPL_) return gemv_launch<ACT_Q8K, LPR_, CPL_, MT_>(ctx, W, w->N, K, w->row_bytes, act, arb, (int)M, y);
    Q8_CASE(4, 1, 4) Q8_CASE(8, 1, 4) Q8_CASE(16, 1, 4) Q8_CASE(32, 1, 4) Q8_CASE(32, 2, 2)
    Q8_CASE(32, 3, 1) Q8_CASE(32, 4, 1)
#undef Q8_CASE
  }
  return set_error(ctx, HAR_CUDA_ERR_UNSUPPORTED, "q4k_gemv: K=" + std::to_string(K) + " exceeds 8192");
}

}  // namespace har
