// k_q6k.cu — Q6_K GEMV on CUDA cores with f32 activations.
//
// Q6_K super-block (210 B, 256 values; the layout q6k_dot reads,
// har/crates/har-demo/src/bin/har-native-qwen3.rs:174-205): ql[128] @0 (low
// nibbles), qh[64] @128 (2-bit high parts), int8 scales[16] @192 (one per 16
// values), f16 d @208.  The value at position half*128 + g*32 + l (half 0..1,
// g 0..3, l 0..31) is d * scales[half*8 + l/16 + 2g] * q with
//   q = (nibble | ((qh[half*32 + l] >> 2g) & 3) << 4) - 32,
// where the nibble is the low half of ql[half*64 + g*32 + l] for g = 0, 1 and
// the high half of ql[half*64 + (g-2)*32 + l] for g = 2, 3.
//
// Work split: one warp per row at a time.  Lane (half, gg, j) = lane bits
// (4, 3, 2..0) owns the 4-byte ql word at 4*lane — ql bytes half*64 + gg*32 +
// 4j..4j+3 — whose low nibbles are group gg and high nibbles group gg+2 of
// positions l = 4j..4j+3, plus the qh word at 128 + half*32 + 4j and the two
// scales it needs.  Rows are 2-byte aligned only (210 B blocks), so words are
// read as two 16-bit loads; each warp load instruction still covers one
// contiguous 128-byte span of the block.  The 6-bit codes are turned into
// floats exactly with a byte permute into the mantissa of 2^23 and one
// subtraction of 2^23 + 32.
//
// Summation order differs from q6k_dot's sequential f32 chain (f32 partial
// sums per lane, then a warp shuffle tree): floating-point parity is the
// path's max-relative-error bound, not bit equality.
#include <algorithm>

#include "har_internal.cuh"
#include "tc_ptx.cuh"

namespace har {

constexpr int Q6K_WARPS = 8;
constexpr int Q6K_BATCH = 4;  // blocks whose words are loaded before any is used

__device__ __forceinline__ uint32_t ld_u16(const uint8_t *p) {
  return __ldg(reinterpret_cast<const unsigned short *>(p));
}

// 6-bit code in byte i of v -> (code - 32) as an exact f32
__device__ __forceinline__ float q6_value(uint32_t v, int i) {
  return __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7440u | (uint32_t)i)) - 8388640.0f;
}

template <int MT>
__global__ void __launch_bounds__(Q6K_WARPS * 32) q6k_gemv_kernel(
    const uint8_t *__restrict__ W, int64_t N, int K, const float *__restrict__ x, int64_t M,
    float *__restrict__ y) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = lane >> 4, gg = (lane >> 3) & 1, ll = (lane & 7) * 4;
  const int ql_off = 4 * lane;
  const int qh_off = 128 + half * 32 + ll;
  const int sc_off = 192 + half * 8 + (ll >> 4) + 2 * gg;
  const int x_off = half * 128 + gg * 32 + ll;
  const int sh_lo = 4 - 2 * gg, sh_hi = 2 * gg;
  const int nb = K / QK;
  const int64_t rb = (int64_t)nb * Q6K_BYTES;
  const int64_t m0 = (int64_t)blockIdx.y * MT;
  const int mt = (int)min((int64_t)MT, M - m0);
  const float *xm = x + m0 * K;

  for (int64_t row = (int64_t)blockIdx.x * Q6K_WARPS + warp; row < N;
       row += (int64_t)gridDim.x * Q6K_WARPS) {
    const uint8_t *r = W + row * rb;
    float acc[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] = 0.0f;
    for (int b0 = 0; b0 < nb; b0 += Q6K_BATCH) {
      uint32_t ql[Q6K_BATCH], qh[Q6K_BATCH], sc[Q6K_BATCH], dh[Q6K_BATCH];
#pragma unroll
      for (int u = 0; u < Q6K_BATCH; ++u) {
        if (b0 + u < nb) {
          const uint8_t *blk = r + (int64_t)(b0 + u) * Q6K_BYTES;
          ql[u] = ld_u16(blk + ql_off) | (ld_u16(blk + ql_off + 2) << 16);
          qh[u] = ld_u16(blk + qh_off) | (ld_u16(blk + qh_off + 2) << 16);
          sc[u] = (uint32_t)__ldg(blk + sc_off) | ((uint32_t)__ldg(blk + sc_off + 4) << 8);
          dh[u] = ld_u16(blk + 208);
        }
      }
#pragma unroll
      for (int u = 0; u < Q6K_BATCH; ++u) {
        if (b0 + u < nb) {
          const uint32_t v0 = (ql[u] & 0x0F0F0F0Fu) | ((qh[u] << sh_lo) & 0x30303030u);
          const uint32_t v1 = ((ql[u] >> 4) & 0x0F0F0F0Fu) | ((qh[u] >> sh_hi) & 0x30303030u);
          const float s0 = (float)(int8_t)(sc[u] & 0xffu);
          const float s1 = (float)(int8_t)(sc[u] >> 8);
          const float d = f16_bits_to_f32(dh[u]);
          float q0[4], q1[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            q0[i] = q6_value(v0, i);
            q1[i] = q6_value(v1, i);
          }
          const float *xb = xm + (int64_t)(b0 + u) * QK + x_off;
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            if (m < mt) {
              const float4 a = __ldg(reinterpret_cast<const float4 *>(xb + (int64_t)m * K));
              const float4 c = __ldg(reinterpret_cast<const float4 *>(xb + (int64_t)m * K + 64));
              float p0 = q0[0] * a.x;
              p0 = fmaf(q0[1], a.y, p0);
              p0 = fmaf(q0[2], a.z, p0);
              p0 = fmaf(q0[3], a.w, p0);
              float p1 = q1[0] * c.x;
              p1 = fmaf(q1[1], c.y, p1);
              p1 = fmaf(q1[2], c.z, p1);
              p1 = fmaf(q1[3], c.w, p1);
              acc[m] = fmaf(d, fmaf(s0, p0, s1 * p1), acc[m]);
            }
          }
        }
      }
    }
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      float v = acc[m];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0 && m < mt) y[(m0 + m) * N + row] = v;
    }
  }
}

// ---------------------------------------------------------------------------
// q6k_gemv_stream_kernel: batch-1 decode when rows are 16-byte aligned (K a
// multiple of 2048).  One CTA per SM owns a contiguous range of rows; one
// producer lane moves stages of Q6S_SR rows (one contiguous byte range each)
// into a ring of shared memory with untiled bulk copies that complete on the
// stage's mbarrier, so the bytes in flight per SM are set by the ring, not by
// registers.  Sixteen compute warps take one row of each stage, read its words
// from shared memory (32-bit loads for the even blocks, which start 4-byte
// aligned, 16-bit pairs for the odd ones), and x from a shared copy.  Every
// wait is bounded; a CTA that gives up sets DEV_ERR_TIMEOUT, waits (bounded)
// for its copies in flight and stops.
// ---------------------------------------------------------------------------
constexpr int Q6S_CW = 16, Q6S_SR = 16, Q6S_MAX_STAGES = 16;
constexpr size_t Q6S_RING = 160 * 1024;
constexpr uint32_t Q6S_WAIT_LIMIT = 1u << 24;

__device__ __forceinline__ bool q6s_wait(uint64_t *bar, uint32_t parity, volatile int *abort_s) {
  for (uint32_t i = 0; i < Q6S_WAIT_LIMIT; ++i) {
    if (tc::mbar_try_wait(bar, parity)) return true;
    if (*abort_s) return false;
  }
  *abort_s = 1;
  return false;
}

__device__ __forceinline__ uint32_t lds_u16(const uint8_t *p) {
  return *reinterpret_cast<const unsigned short *>(p);
}

// One lane's share of one block: d * (s0 * sum_i q0_i x_i + s1 * sum_i q1_i x_i)
__device__ __forceinline__ float q6k_lane_block(uint32_t ql, uint32_t qh, uint32_t sc, uint32_t dh,
                                                int sh_lo, int sh_hi, const float *xb) {
  const uint32_t v0 = (ql & 0x0F0F0F0Fu) | ((qh << sh_lo) & 0x30303030u);
  const uint32_t v1 = ((ql >> 4) & 0x0F0F0F0Fu) | ((qh >> sh_hi) & 0x30303030u);
  const float4 a = *reinterpret_cast<const float4 *>(xb);
  const float4 c = *reinterpret_cast<const float4 *>(xb + 64);
  float p0 = q6_value(v0, 0) * a.x;
  p0 = fmaf(q6_value(v0, 1), a.y, p0);
  p0 = fmaf(q6_value(v0, 2), a.z, p0);
  p0 = fmaf(q6_value(v0, 3), a.w, p0);
  float p1 = q6_value(v1, 0) * c.x;
  p1 = fmaf(q6_value(v1, 1), c.y, p1);
  p1 = fmaf(q6_value(v1, 2), c.z, p1);
  p1 = fmaf(q6_value(v1, 3), c.w, p1);
  const float s0 = (float)(int8_t)(sc & 0xffu), s1 = (float)(int8_t)(sc >> 8);
  return f16_bits_to_f32(dh) * fmaf(s0, p0, s1 * p1);
}

__global__ void __launch_bounds__(32 * (Q6S_CW + 1), 1) q6k_gemv_stream_kernel(
    const uint8_t *__restrict__ W, int64_t N, int K, const float *__restrict__ x,
    float *__restrict__ y, int64_t rows_per_cta, int NS, int *status) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t full[Q6S_MAX_STAGES], empty[Q6S_MAX_STAGES];
  __shared__ volatile int abort_s;
  __shared__ int issued;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = K / QK;
  const int64_t row_bytes = (int64_t)nb * Q6K_BYTES;
  float *xs = reinterpret_cast<float *>(smem);
  uint8_t *ring = smem + (((size_t)K * 4 + 127) & ~(size_t)127);
  const int64_t sb = (int64_t)Q6S_SR * row_bytes;
  const int64_t r_begin = (int64_t)blockIdx.x * rows_per_cta;
  const int64_t r_end = min(N, r_begin + rows_per_cta);
  const int nst = r_end > r_begin ? (int)((r_end - r_begin + Q6S_SR - 1) / Q6S_SR) : 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      tc::mbar_init(full + s, 1);
      tc::mbar_init(empty + s, Q6S_CW);
    }
    abort_s = 0;
    issued = 0;
    tc::fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int s) {
    const int b = s % NS;
    const int64_t r0 = r_begin + (int64_t)s * Q6S_SR;
    const uint32_t bytes = (uint32_t)(min((int64_t)Q6S_SR, r_end - r0) * row_bytes);
    tc::mbar_expect_tx(full + b, bytes);
    tc::bulk_g2s(ring + (int64_t)b * sb, W + r0 * row_bytes, bytes, full + b);
  };
  if (warp == Q6S_CW && lane == 0) {
    for (int s = 0; s < min(NS, nst); ++s) issue(s);
    issued = min(NS, nst);
  }
  for (int i = threadIdx.x; i < K / 4; i += blockDim.x)
    reinterpret_cast<float4 *>(xs)[i] = __ldg(reinterpret_cast<const float4 *>(x) + i);
  __syncthreads();

  if (warp == Q6S_CW) {  // producer: refill each slot once its rows are consumed
    if (lane == 0) {
      for (int s = NS; s < nst; ++s) {
        if (!q6s_wait(empty + s % NS, ((s / NS) & 1u) ^ 1u, &abort_s)) break;
        issue(s);
        issued = s + 1;
      }
    }
  } else {
    const int half = lane >> 4, gg = (lane >> 3) & 1, ll = (lane & 7) * 4;
    const int ql_off = 4 * lane, qh_off = 128 + half * 32 + ll;
    const int sc_off = 192 + half * 8 + (ll >> 4) + 2 * gg;
    const int sh_lo = 4 - 2 * gg, sh_hi = 2 * gg;
    const float *xl = xs + half * 128 + gg * 32 + ll;
    for (int s = 0; s < nst; ++s) {
      const int b = s % NS;
      if (!q6s_wait(full + b, (s / NS) & 1u, &abort_s)) break;
      const int64_t r0 = r_begin + (int64_t)s * Q6S_SR;
      for (int rr = warp; rr < Q6S_SR; rr += Q6S_CW) {
        if (r0 + rr >= r_end) break;
        const uint8_t *row = ring + (int64_t)b * sb + (int64_t)rr * row_bytes;
        float acc = 0.0f;
        for (int k = 0; k < nb; k += 2) {  // nb is even: blocks in (4-aligned, 2-aligned) pairs
          const uint8_t *p0 = row + k * Q6K_BYTES, *p1 = p0 + Q6K_BYTES;
          const uint32_t ql0 = *reinterpret_cast<const uint32_t *>(p0 + ql_off);
          const uint32_t qh0 = *reinterpret_cast<const uint32_t *>(p0 + qh_off);
          const uint32_t ql1 = lds_u16(p1 + ql_off) | (lds_u16(p1 + ql_off + 2) << 16);
          const uint32_t qh1 = lds_u16(p1 + qh_off) | (lds_u16(p1 + qh_off + 2) << 16);
          const uint32_t sc0 = (uint32_t)p0[sc_off] | ((uint32_t)p0[sc_off + 4] << 8);
          const uint32_t sc1 = (uint32_t)p1[sc_off] | ((uint32_t)p1[sc_off + 4] << 8);
          acc += q6k_lane_block(ql0, qh0, sc0, lds_u16(p0 + 208), sh_lo, sh_hi, xl + k * QK);
          acc += q6k_lane_block(ql1, qh1, sc1, lds_u16(p1 + 208), sh_lo, sh_hi, xl + (k + 1) * QK);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) y[r0 + rr] = acc;
      }
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(empty + b);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && abort_s) {
    atomicOr(status, DEV_ERR_TIMEOUT);
    // no exit with a bulk copy into this CTA's shared memory still in flight
    for (int s = max(0, issued - NS); s < issued; ++s)
      tc::mbar_wait(full + s % NS, (s / NS) & 1u, Q6S_WAIT_LIMIT);
  }
}

// The stream kernel's launch, or false when the shape does not suit it.
static bool launch_q6k_stream(har_cuda_ctx *ctx, const uint8_t *W, int64_t N, int K,
                              const float *x, float *y, int32_t *st) {
  const int64_t row_bytes = (int64_t)(K / QK) * Q6K_BYTES;
  if (row_bytes % 16 || ((uintptr_t)W & 15u) || ((uintptr_t)x & 15u)) return false;
  const int64_t sb = (int64_t)Q6S_SR * row_bytes;
  const int NS = (int)std::min<int64_t>(Q6S_MAX_STAGES, (int64_t)Q6S_RING / sb);
  const size_t smem = (((size_t)K * 4 + 127) & ~(size_t)127) + (size_t)NS * (size_t)sb;
  if (NS < 2 || smem > 220 * 1024) return false;
  cudaFuncSetAttribute(q6k_gemv_stream_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       (int)smem);
  const int64_t rows_per_cta = (N + ctx->num_sms - 1) / ctx->num_sms;
  const int64_t grid = (N + rows_per_cta - 1) / rows_per_cta;
  prof_begin(ctx);
  q6k_gemv_stream_kernel<<<(unsigned)grid, 32 * (Q6S_CW + 1), smem, ctx->stream>>>(
      W, N, K, x, y, rows_per_cta, NS, ctx->d_status);
  *st = check_launch(ctx, "q6k_gemv_stream_kernel");
  return true;
}

template <int MT>
static void launch_q6k_mt(har_cuda_ctx *ctx, const uint8_t *W, int64_t N, int K, const float *x,
                          int64_t M, float *y) {
  const int64_t tiles = (M + MT - 1) / MT;
  int64_t gx = (N + Q6K_WARPS - 1) / Q6K_WARPS;
  const int64_t cap = std::max<int64_t>(1, (int64_t)ctx->num_sms * 8 / tiles);
  if (gx > cap) gx = cap;
  q6k_gemv_kernel<MT><<<dim3((unsigned)gx, (unsigned)tiles), Q6K_WARPS * 32, 0, ctx->stream>>>(
      W, N, K, x, M, y);
}

int32_t launch_q6k_gemv(har_cuda_ctx *ctx, const har_cuda_weights *w, int64_t expert,
                        const float *x, int64_t M, float *y) {
  const uint8_t *W = w->dev + expert * w->expert_bytes;
  const int K = (int)w->K;
  int32_t st = HAR_CUDA_OK;
  if (M == 1 && launch_q6k_stream(ctx, W, w->N, K, x, y, &st)) return st;
  prof_begin(ctx);
  if (M == 1)
    launch_q6k_mt<1>(ctx, W, w->N, K, x, M, y);
  else if (M == 2)
    launch_q6k_mt<2>(ctx, W, w->N, K, x, M, y);
  else if (M <= 4)
    launch_q6k_mt<4>(ctx, W, w->N, K, x, M, y);
  else
    launch_q6k_mt<8>(ctx, W, w->N, K, x, M, y);
  return check_launch(ctx, "q6k_gemv_kernel");
}

}  // namespace har
