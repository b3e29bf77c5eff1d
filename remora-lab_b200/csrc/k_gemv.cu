// k_gemv.cu — Q4_K GEMV on CUDA cores for batch-1 and small-M decode:
// y[m][n] = sum_k W_e[n][k] * x[m][k].  Replaces Q4KModel::matvec
// (har/crates/har-serve/src/q4k.rs:170-188), expert_matvec
// (har/crates/har-demo/src/bin/har-native-qwen35moe.rs:626-689) and the
// q4k_gemv / q4k_batched_gemv shaders' role (har/shaders/q4k_gemv.comp,
// har/shaders/q4k_batched_gemv.comp): the same arithmetic, laid out for B200 —
// 128-bit weight loads, activations resident in registers across rows,
// warp-shuffle reduction, MT tokens per weight read.
#include <algorithm>

#include "gemv_engine.cuh"
#include "tc_ptx.cuh"

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

// ---------------------------------------------------------------------------
// Batch-1 decode GEMV with the weights streamed through shared memory.
//
// Each CTA owns a contiguous range of rows, so a stage of SR rows is one
// contiguous byte range: one producer lane moves it with an untiled bulk copy
// (cp.async.bulk, mbarrier transaction count) into a ring of NS stages, and
// CW compute warps take the rows of a stage -- warp w rows w*RPW .. (RPW per
// warp pass, as in q4k_gemv_kernel) -- reading the chunks from shared memory
// with the same arithmetic.  The bytes in flight per SM are then set by the
// ring (about 160 KB), not by how many weight registers the warps hold, which
// is what a streaming GEMV needs to run at HBM rate.  The producer fills the
// whole ring before the activations are staged.  Every wait is bounded; a
// wait that gives up sets DEV_ERR_TIMEOUT and the CTA stops.
// ---------------------------------------------------------------------------
constexpr int GS_MAX_STAGES = 16;
constexpr size_t GS_RING_BYTES = 160 * 1024;
constexpr uint32_t GS_WAIT_LIMIT = 1u << 24;

__device__ __forceinline__ bool gs_wait(uint64_t *bar, uint32_t parity, volatile int *abort_s) {
  for (uint32_t i = 0; i < GS_WAIT_LIMIT; ++i) {
    if (tc::mbar_try_wait(bar, parity)) return true;
    if (*abort_s) return false;
  }
  *abort_s = 1;
  return false;
}

template <int ACT, int LPR, int CPL, int CW>
__global__ void __launch_bounds__(32 * (CW + 1), 1) q4k_gemv_stream_kernel(
    const uint8_t *__restrict__ W, int64_t N, int K, int64_t row_bytes, const uint8_t *__restrict__ act,
    float *__restrict__ y, int64_t rows_per_cta, int NS, int *status) {
  constexpr int RPW = 32 / LPR, SR = CW * RPW;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ const uint8_t *rowp[1];
  __shared__ uint64_t full[GS_MAX_STAGES], empty[GS_MAX_STAGES];
  __shared__ volatile int abort_s;
  __shared__ int issued;  // stages handed to the copy engine
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t act_b = (ActSmem<ACT>::bytes(1, K) + 127) & ~(size_t)127;
  uint8_t *ring = smem + act_b;
  const int64_t sb = (int64_t)SR * row_bytes;  // bytes of a full stage
  const int64_t r_begin = (int64_t)blockIdx.x * rows_per_cta;
  const int64_t r_end = min(N, r_begin + rows_per_cta);
  const int nst = r_end > r_begin ? (int)((r_end - r_begin + SR - 1) / SR) : 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      tc::mbar_init(full + s, 1);
      tc::mbar_init(empty + s, CW);
    }
    abort_s = 0;
    issued = 0;
    rowp[0] = act;
    tc::fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int s) {  // stage s into ring slot s % NS
    const int b = s % NS;
    const int64_t r0 = r_begin + (int64_t)s * SR;
    const uint32_t bytes = (uint32_t)(min((int64_t)SR, r_end - r0) * row_bytes);
    tc::mbar_expect_tx(full + b, bytes);
    tc::bulk_g2s(ring + (int64_t)b * sb, W + r0 * row_bytes, bytes, full + b);
  };
  if (warp == CW && lane == 0) {
    for (int s = 0; s < min(NS, nst); ++s) issue(s);
    issued = min(NS, nst);
  }
  if (ACT == ACT_F32)
    stage_f32(smem, reinterpret_cast<const float *const *>(rowp), 1, K);
  else
    stage_q8k(smem, rowp, 1, K);

  if (warp == CW) {  // producer: refill each slot once its rows are consumed
    if (lane == 0) {
      for (int s = NS; s < nst; ++s) {
        if (!gs_wait(empty + s % NS, ((s / NS) & 1u) ^ 1u, &abort_s)) break;
        issue(s);
        issued = s + 1;
      }
    }
  } else {
    const int grp = lane / LPR, gl = lane % LPR;
    const int C = K / 64;
    LaneAct<ACT> a[CPL];
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      const int ch = gl + LPR * i;
      if (ch < C) a[i].load(smem, 1, K, 0, ch);
    }
    for (int s = 0; s < nst; ++s) {
      const int b = s % NS;
      if (!gs_wait(full + b, (s / NS) & 1u, &abort_s)) break;
      const int64_t r0 = r_begin + (int64_t)s * SR;
      const int rr = warp * RPW + grp;  // row of this lane group in the stage
      const bool valid = r0 + rr < r_end;
      const uint8_t *row = ring + (int64_t)b * sb + (int64_t)(valid ? rr : 0) * row_bytes;
      float acc = 0.0f;
#pragma unroll
      for (int i = 0; i < CPL; ++i) {
        const int ch = gl + LPR * i;
        if (ch < C) acc += chunk_dot(load_wchunk_s(row, ch), ch, a[i]);
      }
      acc = lane_group_sum<LPR>(acc);
      if (valid && gl == 0) y[r0 + rr] = acc;
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(empty + b);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && abort_s) {
    atomicOr(status, DEV_ERR_TIMEOUT);
    // A CTA that stopped early must not exit with a bulk copy into its shared
    // memory still in flight: wait (bounded) for the last stage issued into
    // each slot; the earlier ones completed before the slot was reused.
    for (int s = max(0, issued - NS); s < issued; ++s) tc::mbar_wait(full + s % NS, (s / NS) & 1u, GS_WAIT_LIMIT);
  }
}

template <int ACT, int LPR, int CPL, int CW>
static int32_t gemv_stream_launch(har_cuda_ctx *ctx, const uint8_t *W, int64_t N, int K,
                                  int64_t row_bytes, const uint8_t *act, float *y) {
  constexpr int RPW = 32 / LPR, SR = CW * RPW;
  auto kern = q4k_gemv_stream_kernel<ACT, LPR, CPL, CW>;
  const int64_t sb = (int64_t)SR * row_bytes;
  const int NS = (int)std::max<int64_t>(2, std::min<int64_t>(GS_MAX_STAGES, (int64_t)GS_RING_BYTES / sb));
  const size_t act_b = (ActSmem<ACT>::bytes(1, K) + 127) & ~(size_t)127;
  const size_t smem = act_b + (size_t)NS * (size_t)sb + 128;
  if (smem > 220 * 1024) return set_error(ctx, HAR_CUDA_ERR_UNSUPPORTED, "q4k_gemv: K too large");
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  // one CTA per SM (a CTA's last stage may hold fewer than SR rows)
  const int64_t rows_per_cta = (N + ctx->num_sms - 1) / ctx->num_sms;
  const int64_t grid = (N + rows_per_cta - 1) / rows_per_cta;
  prof_begin(ctx);
  kern<<<(unsigned)grid, 32 * (CW + 1), smem, ctx->stream>>>(W, N, K, row_bytes, act, y, rows_per_cta, NS,
                                                              ctx->d_status);
  return check_launch(ctx, "q4k_gemv_stream_kernel");
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
    if (M == 1) {  // decode: weights streamed through shared memory
#define F32_S_CASE(LPR_, CPL_) \
  if (s.LPR == LPR_ && s.CPL == CPL_) return gemv_stream_launch<ACT_F32, LPR_, CPL_, 8>(ctx, W, w->N, K, w->row_bytes, act, y);
      // (K > 4096 keeps the register-resident kernel: 64 f32 activations per chunk
      // and lane do not fit beside a stream of rows)
      F32_S_CASE(4, 1) F32_S_CASE(8, 1) F32_S_CASE(16, 1) F32_S_CASE(32, 1) F32_S_CASE(32, 2)
#undef F32_S_CASE
    }
    const int64_t arb = (int64_t)K * 4;
#define F32_CASE(LPR_, CPL_) \
  if (s.LPR == LPR_ && s.CPL == CPL_) return gemv_launch<ACT_F32, LPR_, CPL_, 1>(ctx, W, w->N, K, w->row_bytes, act, arb, (int)M, y);
    F32_CASE(4, 1) F32_CASE(8, 1) F32_CASE(16, 1) F32_CASE(32, 1) F32_CASE(32, 2)
    F32_CASE(32, 3) F32_CASE(32, 4)
#undef F32_CASE
  } else {
    if ((uintptr_t)x & 3u) return set_error(ctx, HAR_CUDA_ERR_ARG, "q4k_gemv: Q8_K rows must be 4-byte aligned");
    if (M == 1) {
#define Q8_S_CASE(LPR_, CPL_) \
  if (s.LPR == LPR_ && s.CPL == CPL_) return gemv_stream_launch<ACT_Q8K, LPR_, CPL_, 16>(ctx, W, w->N, K, w->row_bytes, act, y);
      Q8_S_CASE(4, 1) Q8_S_CASE(8, 1) Q8_S_CASE(16, 1) Q8_S_CASE(32, 1) Q8_S_CASE(32, 2)
      Q8_S_CASE(32, 3) Q8_S_CASE(32, 4)
#undef Q8_S_CASE
    }
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
