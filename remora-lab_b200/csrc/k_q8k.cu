// k_q8k.cu — Q8_K activation quantisation (one warp per 256-value block).
//
// Block format (292 B): f32 d @0, int8 qs[256] @4, int16 bsums[16] @260.
//   amax = max |x|; amax == 0 -> d = 0, qs = 0;
//   iscale = 127/amax (IEEE division), q = clamp(rint(x*iscale), -127, 127)
//   (when 127/amax overflows to inf: q = clamp(rint(x/d), -127, 127)),
//   d = amax/127; bsums[g] = sum of qs[16g .. 16g+15].
// Every step is a correctly rounded IEEE operation or exact integer work, so
// the result is bit-identical to the CPU restatement (oracle/har_oracle.c,
// haro_q8k_quantize).  The reference has no Q8_K quantiser; its geometry
// (292 B / 256 values) is recorded at
// benchmarks/local-bench/crates/lb-model/src/lib.rs:88.
#include "har_internal.cuh"

namespace har {

__device__ __forceinline__ int q8_of(float x, float iscale, float d, bool use_div) {
  const float t = use_div ? __fdiv_rn(x, d) : __fmul_rn(x, iscale);
  return max(-127, min(127, __float2int_rn(t)));
}

__global__ void __launch_bounds__(256) q8k_quantize_kernel(const float *__restrict__ x,
                                                           int64_t nblocks,
                                                           uint8_t *__restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t blk = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (blk >= nblocks) return;
  const float4 *src = reinterpret_cast<const float4 *>(x + blk * QK + lane * 8);
  float4 a = src[0], b = src[1];
  float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  int q[8];
  float d = 0.0f;
  if (amax == 0.0f) {
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] = 0;
  } else {
    const float iscale = __fdiv_rn(127.0f, amax);
    d = __fdiv_rn(amax, 127.0f);
    const bool use_div = isinf(iscale);  // amax below 127/FLT_MAX
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] = q8_of(v[i], iscale, d, use_div);
  }
  int s = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) s += q[i];
  s += __shfl_xor_sync(0xffffffffu, s, 1);  // lanes 2g, 2g+1 hold values 16g..16g+15
  uint8_t *o = out + blk * Q8K_BYTES;
  uint32_t w0 = (uint32_t)(q[0] & 0xff) | ((uint32_t)(q[1] & 0xff) << 8) |
                ((uint32_t)(q[2] & 0xff) << 16) | ((uint32_t)(q[3] & 0xff) << 24);
  uint32_t w1 = (uint32_t)(q[4] & 0xff) | ((uint32_t)(q[5] & 0xff) << 8) |
                ((uint32_t)(q[6] & 0xff) << 16) | ((uint32_t)(q[7] & 0xff) << 24);
  reinterpret_cast<uint32_t *>(o + 4 + 8 * lane)[0] = w0;
  reinterpret_cast<uint32_t *>(o + 4 + 8 * lane)[1] = w1;
  if ((lane & 1) == 0) reinterpret_cast<int16_t *>(o + 260)[lane >> 1] = (int16_t)s;
  if (lane == 0) *reinterpret_cast<float *>(o) = d;
}

int32_t launch_q8k_quantize(har_cuda_ctx *ctx, const float *x, int64_t M, int64_t K,
                            uint8_t *out) {
  if (((uintptr_t)x & 15u) || ((uintptr_t)out & 3u))
    return set_error(ctx, HAR_CUDA_ERR_ARG,
                     "q8k_quantize: x must be 16-byte and out 4-byte aligned");
  const int64_t nblocks = M * (K / QK);
  const int64_t grid = (nblocks + 7) / 8;
  prof_begin(ctx);
  q8k_quantize_kernel<<<(unsigned)grid, 256, 0, ctx->stream>>>(x, nblocks, out);
  return check_launch(ctx, "q8k_quantize_kernel");
}

}  // namespace har
