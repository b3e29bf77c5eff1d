// k_gen.cu — synthetic Q4_K weights generated on the device (bench/test input
// generator; not a reference function).  The formula is the oracle's
// (oracle/har_oracle.c: haro_normal_at + haro_q4k_quantize_block): value i of
// a seed is a Box-Muller normal from two splitmix64 words of (seed, i/2),
// scaled to N(mean, std) and rounded to f32; each 256-value block is then
// quantised by the same sequence of correctly rounded f32 operations, so a
// block is byte-identical to the host generator's whenever the double-precision
// log/sin/cos of the two libraries round the same way (almost always).
// One warp per super-block; lane l holds values 8l .. 8l+7.
#include <algorithm>

#include "har_internal.cuh"

namespace har {

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
  return z ^ (z >> 31);
}

__device__ __forceinline__ double normal_at(uint64_t seed, int64_t i) {
  const uint64_t pp = (uint64_t)(i >> 1);
  const uint64_t base = seed * 0x9E3779B97F4A7C15ULL;
  const uint64_t a = mix64(base + 2 * pp + 1);
  const uint64_t b = mix64(base + 2 * pp + 2);
  const double u1 = (double)((a >> 11) + 1) * (1.0 / 9007199254740992.0);
  const double u2 = (double)(b >> 11) * (1.0 / 9007199254740992.0);
  const double r = sqrt(-2.0 * log(u1));
  const double th = 6.283185307179586 * u2;
  return (i & 1) ? r * sin(th) : r * cos(th);
}

__global__ void __launch_bounds__(256) gen_q4k_kernel(uint8_t *__restrict__ dst, int64_t nblk,
                                                      int64_t bpr, int64_t K, uint64_t seed,
                                                      int64_t row0, float mean, float stdv) {
  const int lane = threadIdx.x & 31;
  const int64_t blk = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (blk >= nblk) return;
  const int64_t r = blk / bpr, b = blk - r * bpr;
  const int64_t first = (row0 + r) * K + b * QK + 8 * lane;
  float v[8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
    v[i] = (float)((double)mean + (double)stdv * normal_at(seed, first + i));
  // sub-block j = lane/4: min / max over its 4 lanes
  float lo = v[0], hi = v[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) {
    lo = fminf(lo, v[i]);
    hi = fmaxf(hi, v[i]);
  }
#pragma unroll
  for (int o = 1; o < 4; o <<= 1) {
    lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  if (lo > 0.0f) lo = 0.0f;
  const float scale = __fdiv_rn(__fsub_rn(hi, lo), 15.0f);
  const float off = -lo;
  float smax = scale, omax = off;
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    smax = fmaxf(smax, __shfl_xor_sync(0xffffffffu, smax, o));
    omax = fmaxf(omax, __shfl_xor_sync(0xffffffffu, omax, o));
  }
  const __half dh = __float2half_rn(__fdiv_rn(smax, 63.0f));
  const __half mh = __float2half_rn(__fdiv_rn(omax, 63.0f));
  const float df = __half2float(dh), mf = __half2float(mh);
  const int sc = df > 0.0f ? max(0, min(63, (int)rintf(__fdiv_rn(scale, df)))) : 0;
  const int mn = mf > 0.0f ? max(0, min(63, (int)rintf(__fdiv_rn(off, mf)))) : 0;
  const float step = __fmul_rn(df, (float)sc);
  const float bias = __fmul_rn(mf, (float)mn);
  uint32_t nib[2] = {0u, 0u};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int q = step > 0.0f ? max(0, min(15, (int)rintf(__fdiv_rn(__fadd_rn(v[i], bias), step)))) : 0;
    nib[i >> 2] |= (uint32_t)q << (8 * (i & 3));
  }
  // pair sub-blocks 2c (low nibbles) and 2c+1 (high nibbles): lane l (j even)
  // takes lane l+4's nibbles.
  const uint32_t up0 = __shfl_down_sync(0xffffffffu, nib[0], 4);
  const uint32_t up1 = __shfl_down_sync(0xffffffffu, nib[1], 4);
  // scale bytes: gather the 8 (sc, m) pairs onto every lane
  int scs[8], mns[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    scs[j] = __shfl_sync(0xffffffffu, sc, 4 * j);
    mns[j] = __shfl_sync(0xffffffffu, mn, 4 * j);
  }
  uint8_t *o = dst + blk * Q4K_BYTES;
  const int j = lane >> 2;
  if ((j & 1) == 0) {
    uint32_t *w = reinterpret_cast<uint32_t *>(o + 16 + (j >> 1) * 32 + (lane & 3) * 8);
    w[0] = nib[0] | (up0 << 4);
    w[1] = nib[1] | (up1 << 4);
  }
  if (lane == 0) {
    uint32_t hdr[4];
    hdr[0] = (uint32_t)__half_as_ushort(dh) | ((uint32_t)__half_as_ushort(mh) << 16);
    uint8_t s[12];
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      s[jj] = (uint8_t)((scs[jj] & 63) | ((scs[jj + 4] >> 4) << 6));
      s[jj + 4] = (uint8_t)((mns[jj] & 63) | ((mns[jj + 4] >> 4) << 6));
      s[jj + 8] = (uint8_t)((scs[jj + 4] & 15) | ((mns[jj + 4] & 15) << 4));
    }
#pragma unroll
    for (int w = 0; w < 3; ++w)
      hdr[1 + w] = (uint32_t)s[4 * w] | ((uint32_t)s[4 * w + 1] << 8) |
                   ((uint32_t)s[4 * w + 2] << 16) | ((uint32_t)s[4 * w + 3] << 24);
    *reinterpret_cast<uint4 *>(o) = make_uint4(hdr[0], hdr[1], hdr[2], hdr[3]);
  }
}

int32_t launch_gen_q4k(har_cuda_ctx *ctx, uint8_t *dst, int64_t rows, int64_t K,
                       uint64_t seed, int64_t row0, float mean, float stdv) {
  if ((uintptr_t)dst & 15u) return set_error(ctx, HAR_CUDA_ERR_ARG, "gen_q4k: dst must be 16-byte aligned");
  const int64_t bpr = K / QK;
  const int64_t nblk = rows * bpr;
  (void)nblk;
  // launches of whole rows, at most ~2^24 super-blocks each
  const int64_t rows_per_launch = std::max<int64_t>(1, ((int64_t)1 << 24) / bpr);
  for (int64_t r0 = 0; r0 < rows; r0 += rows_per_launch) {
    const int64_t nrows = std::min<int64_t>(rows_per_launch, rows - r0);
    const int64_t nbl = nrows * bpr;
    prof_begin(ctx);
    gen_q4k_kernel<<<(unsigned)((nbl + 7) / 8), 256, 0, ctx->stream>>>(
        dst + r0 * bpr * Q4K_BYTES, nbl, bpr, K, seed, row0 + r0, mean, stdv);
    int32_t st = check_launch(ctx, "gen_q4k_kernel");
    if (st) return st;
  }
  return HAR_CUDA_OK;
}

}  // namespace har
