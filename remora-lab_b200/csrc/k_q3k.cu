// k_q3k.cu — Q3_K GEMV on CUDA cores with f32 activations.
//
// Q3_K super-block (110 B, 256 values; GGML type 11, the geometry the
// reference records at har/crates/har-model/src/lib.rs:591 and
// benchmarks/local-bench/crates/lb-model/src/lib.rs:84 — it has no Q3_K
// arithmetic, so the layout is GGUF's as ggml defines it): hmask[32] @0,
// qs[64] @32 (2-bit planes), 12 bytes of packed 6-bit scales @96, f16 d @108.
// Value i = 128n + 32j + l (n < 2, j < 4, l < 32) is
//   d * (scale[8n + 2j + l/16] - 32) * (((qs[32n + l] >> 2j) & 3) + 4 * hbit - 4),
//   hbit = (hmask[l] >> (4n + j)) & 1;
// scale s keeps its low four bits in byte s & 7 (low nibble for s < 8, high
// nibble above) and its top two bits in byte 8 + s % 4 at bit 2 * (s / 4).
//
// Work split: one warp per row at a time.  Lane (n, jh, a) = lane bits
// (4, 3, 2..0) owns positions l = 4a..4a+3 of planes j = 2jh and 2jh + 1 in
// half n: the qs word at 32 + 32n + 4a, the hmask word at 4a, and the two
// scales of sub-blocks 8n + 4jh + a/4 (+2).  A 3-bit code goes to an exact
// f32 by a byte permute into the mantissa of 2^23 and one subtraction of
// 2^23 + 4.  Blocks are 2-byte aligned only, so words are read as two 16-bit
// loads; several blocks' words are loaded before any is used.
//
// Summation order: per lane, per plane, four products left to right, scaled
// by the plane's sub-block scale and d, then a warp shuffle tree — not the
// oracle's sequential chain, so parity is a max-relative-error bound.
#include <algorithm>

#include "har_internal.cuh"
#include "tc_ptx.cuh"

namespace har {

constexpr int Q3K_WARPS = 8;
constexpr int Q3K_BATCH = 4;  // blocks whose words are loaded before any is used

__device__ __forceinline__ uint32_t q3_ld_u16(const uint8_t *p) {
  return __ldg(reinterpret_cast<const unsigned short *>(p));
}

// 3-bit code in byte i of v -> (code - 4) as an exact f32
__device__ __forceinline__ float q3_value(uint32_t v, int i) {
  return __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7440u | (uint32_t)i)) - 8388612.0f;
}

struct Q3Lane {
  int n, jh, a;
  int qs_off, hm_off, lo0, lo1, hi0, hi1, lo_shift, hi_shift, pl0;  // byte offsets and shifts
  int x_off;
};

__device__ __forceinline__ Q3Lane q3_lane(int lane) {
  Q3Lane L;
  L.n = lane >> 4;
  L.jh = (lane >> 3) & 1;
  L.a = lane & 7;
  L.qs_off = 32 + 32 * L.n + 4 * L.a;
  L.hm_off = 4 * L.a;
  L.lo0 = 96 + 4 * L.jh + (L.a >> 2);  // low-nibble bytes of sub-blocks s0 and s0 + 2
  L.lo1 = L.lo0 + 2;
  L.hi0 = 96 + 8 + (L.a >> 2);  // top-bit bytes of the same two
  L.hi1 = L.hi0 + 2;
  L.lo_shift = 4 * L.n;
  L.hi_shift = 2 * (2 * L.n + L.jh);
  L.pl0 = 2 * L.jh;  // plane j of the lane's first group
  L.x_off = 128 * L.n + 32 * L.pl0 + 4 * L.a;
  return L;
}

// (scale0 - 32, scale1 - 32) from the four scale bytes (lo0, lo1, hi0, hi1 packed low to high)
__device__ __forceinline__ float2 q3_scales(uint32_t sb, const Q3Lane &L) {
  const uint32_t s0 = ((sb >> L.lo_shift) & 15u) | (((sb >> (16 + L.hi_shift)) & 3u) << 4);
  const uint32_t s1 = ((sb >> (8 + L.lo_shift)) & 15u) | (((sb >> (24 + L.hi_shift)) & 3u) << 4);
  return make_float2((float)((int)s0 - 32), (float)((int)s1 - 32));
}

// codes of planes pl0 and pl0 + 1 at the lane's four positions, one per byte
__device__ __forceinline__ void q3_codes(uint32_t qs, uint32_t hm, const Q3Lane &L, uint32_t &c0,
                                         uint32_t &c1) {
  const int j0 = L.pl0, hb = 4 * L.n + j0;
  c0 = ((qs >> (2 * j0)) & 0x03030303u) | (((hm >> hb) & 0x01010101u) << 2);
  c1 = ((qs >> (2 * j0 + 2)) & 0x03030303u) | (((hm >> (hb + 1)) & 0x01010101u) << 2);
}

template <int MT>
__global__ void __launch_bounds__(Q3K_WARPS * 32) q3k_gemv_kernel(
    const uint8_t *__restrict__ W, int64_t N, int K, const float *__restrict__ x, int64_t M,
    float *__restrict__ y) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const Q3Lane L = q3_lane(lane);
  const int nb = K / QK;
  const int64_t rb = (int64_t)nb * Q3K_BYTES;
  const int64_t m0 = (int64_t)blockIdx.y * MT;
  const int mt = (int)min((int64_t)MT, M - m0);
  const float *xm = x + m0 * K;

  for (int64_t row = (int64_t)blockIdx.x * Q3K_WARPS + warp; row < N;
       row += (int64_t)gridDim.x * Q3K_WARPS) {
    const uint8_t *r = W + row * rb;
    float acc[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] = 0.0f;
    for (int b0 = 0; b0 < nb; b0 += Q3K_BATCH) {
      uint32_t qs[Q3K_BATCH], hm[Q3K_BATCH], sb[Q3K_BATCH], dh[Q3K_BATCH];
#pragma unroll
      for (int u = 0; u < Q3K_BATCH; ++u) {
        if (b0 + u < nb) {
          const uint8_t *blk = r + (int64_t)(b0 + u) * Q3K_BYTES;
          qs[u] = q3_ld_u16(blk + L.qs_off) | (q3_ld_u16(blk + L.qs_off + 2) << 16);
          hm[u] = q3_ld_u16(blk + L.hm_off) | (q3_ld_u16(blk + L.hm_off + 2) << 16);
          sb[u] = (uint32_t)__ldg(blk + L.lo0) | ((uint32_t)__ldg(blk + L.lo1) << 8) |
                  ((uint32_t)__ldg(blk + L.hi0) << 16) | ((uint32_t)__ldg(blk + L.hi1) << 24);
          dh[u] = q3_ld_u16(blk + 108);
        }
      }
#pragma unroll
      for (int u = 0; u < Q3K_BATCH; ++u) {
        if (b0 + u < nb) {
          uint32_t c0, c1;
          q3_codes(qs[u], hm[u], L, c0, c1);
          const float2 s = q3_scales(sb[u], L);
          const float d = f16_bits_to_f32(dh[u]);
          float q0[4], q1[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            q0[i] = q3_value(c0, i);
            q1[i] = q3_value(c1, i);
          }
          const float *xb = xm + (int64_t)(b0 + u) * QK + L.x_off;
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            if (m < mt) {
              const float4 xa = __ldg(reinterpret_cast<const float4 *>(xb + (int64_t)m * K));
              const float4 xc = __ldg(reinterpret_cast<const float4 *>(xb + (int64_t)m * K + 32));
              float p0 = q0[0] * xa.x;
              p0 = fmaf(q0[1], xa.y, p0);
              p0 = fmaf(q0[2], xa.z, p0);
              p0 = fmaf(q0[3], xa.w, p0);
              float p1 = q1[0] * xc.x;
              p1 = fmaf(q1[1], xc.y, p1);
              p1 = fmaf(q1[2], xc.z, p1);
              p1 = fmaf(q1[3], xc.w, p1);
              acc[m] = fmaf(d, fmaf(s.x, p0, s.y * p1), acc[m]);
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
// q3k_gemv_smem_kernel: the same lane split with each warp's rows staged in
// shared memory.  Global loads of 16-bit fields from 2-byte-aligned 110-byte
// blocks spread one warp instruction over several sectors; here each warp
// copies whole rows (row bytes a multiple of 16) with 16-byte cp.async,
// double-buffered — the next row is in flight while the current one is
// computed — and the lanes read their fields from shared memory.
// Lane split: half-warp hw takes block b + hw of each pair of blocks; lane
// (n, a) of a half owns positions l = 4a..4a+3 of half n in all four planes
// (16 values): one qs word, one hmask word, the four sub-block scales of
// those positions (low nibbles in bytes a/4 + 2j, top bits in bytes
// 8 + a/4 and 10 + a/4), so each value costs fewer shared-memory loads than
// the 8-value split.  Codes become exact f32 by a byte permute into the
// mantissa of 2^23; the offset and the products run as packed f32x2.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t q3_lds_u16(const uint8_t *p) {
  return *reinterpret_cast<const unsigned short *>(p);
}

template <int MT>
__global__ void __launch_bounds__(Q3K_WARPS * 32) q3k_gemv_smem_kernel(
    const uint8_t *__restrict__ W, int64_t N, int K, const float *__restrict__ x, int64_t M,
    float *__restrict__ y) {
  extern __shared__ __align__(16) uint8_t q3s[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = K / QK;
  const int rb = nb * Q3K_BYTES;  // a multiple of 16 (the launcher checks)
  uint8_t *const base = q3s + (size_t)warp * 2 * rb;  // this warp's two row buffers
  const int hw = lane >> 4, n = (lane >> 3) & 1, a = lane & 7, c = a >> 2;
  const int qs_off = 32 + 32 * n + 4 * a, hm_off = 4 * a, x_off = 128 * n + 4 * a;
  const int64_t m0 = (int64_t)blockIdx.y * MT;
  const int mt = (int)min((int64_t)MT, M - m0);
  const float *xm = x + m0 * K;
  const int64_t stride = (int64_t)gridDim.x * Q3K_WARPS;
  auto issue = [&](int64_t row, uint8_t *dst) {  // one commit group per row (empty past the end)
    if (row < N) {
      const uint8_t *src = W + row * (int64_t)rb;
      for (int i = lane; i < rb / 16; i += 32) tc::cp_async16(dst + 16 * i, src + 16 * i, 16u);
    }
    tc::cp_async_commit();
  };
  int64_t row = (int64_t)blockIdx.x * Q3K_WARPS + warp;
  issue(row, base);
  for (int cur = 0; row < N; row += stride, cur ^= 1) {
    issue(row + stride, base + (cur ^ 1) * rb);
    tc::cp_async_wait<1>();  // this lane's copies of the current row
    __syncwarp();            // ... and every other lane's
    const uint8_t *r = base + cur * rb;
    float acc[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] = 0.0f;
#pragma unroll 2
    for (int b = hw; b < nb; b += 2) {  // nb is even here (rows are a multiple of 16 bytes)
      const uint8_t *blk = r + b * Q3K_BYTES;
      const uint32_t qs = q3_lds_u16(blk + qs_off) | (q3_lds_u16(blk + qs_off + 2) << 16);
      const uint32_t hm = q3_lds_u16(blk + hm_off) | (q3_lds_u16(blk + hm_off + 2) << 16);
      const uint32_t top0 = blk[96 + 8 + c], top1 = blk[96 + 10 + c];
      const float d = f16_bits_to_f32(q3_lds_u16(blk + 108));
      float2 q[4][2];  // plane j: positions (0, 1), (2, 3) as code - 4
      float sc[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t low = blk[96 + c + 2 * j];
        const uint32_t top = (j & 1) ? top1 : top0;
        sc[j] = (float)((int)(((low >> (4 * n)) & 15u) | (((top >> (4 * n + 2 * (j >> 1))) & 3u) << 4)) - 32);
        const uint32_t code = ((qs >> (2 * j)) & 0x03030303u) | (((hm >> (4 * n + j)) & 0x01010101u) << 2);
        const float2 lo = make_float2(__uint_as_float(__byte_perm(code, 0x4B000000u, 0x7440u)),
                                      __uint_as_float(__byte_perm(code, 0x4B000000u, 0x7441u)));
        const float2 hi = make_float2(__uint_as_float(__byte_perm(code, 0x4B000000u, 0x7442u)),
                                      __uint_as_float(__byte_perm(code, 0x4B000000u, 0x7443u)));
        q[j][0] = __fadd2_rn(lo, make_float2(-8388612.0f, -8388612.0f));
        q[j][1] = __fadd2_rn(hi, make_float2(-8388612.0f, -8388612.0f));
      }
      const float *xb = xm + (int64_t)b * QK + x_off;
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        if (m < mt) {
          float sum = 0.0f;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float4 xv = __ldg(reinterpret_cast<const float4 *>(xb + (int64_t)m * K + 32 * j));
            float2 p = __fmul2_rn(q[j][0], make_float2(xv.x, xv.y));
            p = __ffma2_rn(q[j][1], make_float2(xv.z, xv.w), p);
            sum = fmaf(sc[j], p.x + p.y, sum);
          }
          acc[m] = fmaf(d, sum, acc[m]);
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
    __syncwarp();  // every lane is done with this buffer before the next issue refills it
  }
  tc::cp_async_wait<0>();
}

// Shared memory of the staged kernel (two rows per warp), or 0 when the
// shape does not suit it (row bytes not a multiple of 16, too long a row,
// an unaligned base).
static size_t q3k_smem_bytes(int K, const uint8_t *W) {
  const size_t rb = (size_t)(K / QK) * Q3K_BYTES;
  if (rb % 16 || ((uintptr_t)W & 15u)) return 0;
  const size_t bytes = 2 * Q3K_WARPS * rb;
  return bytes <= 200 * 1024 ? bytes : 0;
}

template <int MT>
static void launch_q3k_smem(har_cuda_ctx *ctx, const uint8_t *W, int64_t N, int K, const float *x,
                            int64_t M, float *y, size_t smem) {
  cudaFuncSetAttribute(q3k_gemv_smem_kernel<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int64_t tiles = (M + MT - 1) / MT;
  int64_t gx = (N + Q3K_WARPS - 1) / Q3K_WARPS;
  const int64_t cap = std::max<int64_t>(1, (int64_t)ctx->num_sms * 8 / tiles);
  if (gx > cap) gx = cap;
  q3k_gemv_smem_kernel<MT><<<dim3((unsigned)gx, (unsigned)tiles), Q3K_WARPS * 32, smem, ctx->stream>>>(
      W, N, K, x, M, y);
}

template <int MT>
static void launch_q3k_mt(har_cuda_ctx *ctx, const uint8_t *W, int64_t N, int K, const float *x,
                          int64_t M, float *y) {
  const int64_t tiles = (M + MT - 1) / MT;
  int64_t gx = (N + Q3K_WARPS - 1) / Q3K_WARPS;
  const int64_t cap = std::max<int64_t>(1, (int64_t)ctx->num_sms * 8 / tiles);
  if (gx > cap) gx = cap;
  q3k_gemv_kernel<MT><<<dim3((unsigned)gx, (unsigned)tiles), Q3K_WARPS * 32, 0, ctx->stream>>>(
      W, N, K, x, M, y);
}

int32_t launch_q3k_gemv(har_cuda_ctx *ctx, const har_cuda_weights *w, int64_t expert,
                        const float *x, int64_t M, float *y) {
  const uint8_t *W = w->dev + expert * w->expert_bytes;
  const int K = (int)w->K;
  prof_begin(ctx);
  const size_t smem = q3k_smem_bytes(K, W);
  if (smem) {
    if (M == 1)
      launch_q3k_smem<1>(ctx, W, w->N, K, x, M, y, smem);
    else if (M == 2)
      launch_q3k_smem<2>(ctx, W, w->N, K, x, M, y, smem);
    else if (M <= 4)
      launch_q3k_smem<4>(ctx, W, w->N, K, x, M, y, smem);
    else
      launch_q3k_smem<8>(ctx, W, w->N, K, x, M, y, smem);
    return check_launch(ctx, "q3k_gemv_smem_kernel");
  }
  if (M == 1)
    launch_q3k_mt<1>(ctx, W, w->N, K, x, M, y);
  else if (M == 2)
    launch_q3k_mt<2>(ctx, W, w->N, K, x, M, y);
  else if (M <= 4)
    launch_q3k_mt<4>(ctx, W, w->N, K, x, M, y);
  else
    launch_q3k_mt<8>(ctx, W, w->N, K, x, M, y);
  return check_launch(ctx, "q3k_gemv_kernel");
}

}  // namespace har
