// har_internal.cuh — shared device helpers and host-side handle types of
// libhar_cuda.so.  Q4_K semantics follow har/crates/har-serve/src/q4k.rs:12-89
// and har/crates/har-demo/src/bin/har-native-qwen3.rs:116-172 (paths relative
// to the leoinfer/remora-lab repository).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "har_cuda.h"

namespace har {

constexpr int QK = 256;           // values per super-block
constexpr int Q4K_BYTES = 144;    // bytes per Q4_K super-block
constexpr int Q6K_BYTES = 210;    // bytes per Q6_K super-block
constexpr int Q3K_BYTES = 110;    // bytes per Q3_K super-block
// GGML tensor type ids (the ids HAR's GGUF reader matches,
// har/crates/har-demo/src/bin/har-native-qwen35moe.rs:37-41; Q3_K's from
// har/crates/har-model/src/lib.rs:591)
constexpr int GGML_F32 = 0, GGML_Q3_K = 11, GGML_Q4_K = 12, GGML_Q6_K = 14;
// bytes per 256-value super-block of the block types the weights accept (0 = other)
inline int ggml_block_bytes(int type) {
  return type == GGML_Q4_K ? Q4K_BYTES : type == GGML_Q6_K ? Q6K_BYTES : type == GGML_Q3_K ? Q3K_BYTES : 0;
}
constexpr int Q8K_BYTES = 292;    // bytes per Q8_K block
constexpr float ROUTER_EPS = 1.0e-9f;

// Device error words (bit flags) written by kernels; read by har_cuda_synchronize.
constexpr int DEV_ERR_TIMEOUT = 1;
constexpr int DEV_ERR_BOUNDS = 2;
// a value outside the tensor-core path's range: an activation, a sub-block sum
// of activations or a SwiGLU output of magnitude >= 65520 (f16 overflows), or
// a Q4_K block whose min offset exceeds 2^29 times its scale step; the call's
// results are not valid (the CUDA-core path, HAR_CUDA_MOE_FORCE_GEMV, has no
// such limit)
constexpr int DEV_ERR_RANGE = 4;

// ---------------------------------------------------------------------------
// Q4_K super-block header: 16 bytes = {d|dmin<<16, sc/m bytes 0-3, 4-7, 8-11}
// ---------------------------------------------------------------------------

__device__ __forceinline__ float f16_bits_to_f32(uint32_t bits16) {
  // binary16 -> f32 is exact (subnormals included): the same value as
  // f16_to_f32 (q4k.rs:22-50) and half_to_f32 (har-native-qwen3.rs:116-136).
  return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xffffu)));
}

// 6-bit scale and min of sub-block j (0..7) from the three scale words
// s0 = bytes 4..7, s1 = bytes 8..11, s2 = bytes 12..15 of the block
// (scale_min, har-native-qwen3.rs:138-147; scale_at/min_at, q4k.rs:60-74).
__device__ __forceinline__ void q4k_scale_min(uint32_t s0, uint32_t s1, uint32_t s2, int j,
                                              int &sc, int &m) {
  if (j < 4) {
    sc = (s0 >> (8 * j)) & 63;
    m = (s1 >> (8 * j)) & 63;
  } else {
    const int b = 8 * (j - 4);
    const uint32_t lo = (s2 >> b) & 0xffu;
    sc = (lo & 15) | (((s0 >> b) >> 6 & 3) << 4);
    m = (lo >> 4) | (((s1 >> b) >> 6 & 3) << 4);
  }
}

// Dequantised f32 value pair constants of a 64-value chunk c (sub-blocks 2c, 2c+1):
// value = d1 * q - m1 for the low nibble half, d2 * q - m2 for the high half.
struct ChunkScales {
  float d1, m1, d2, m2;  // d*sc, dmin*m  (q4k_dot's d1/min1/d2/min2)
  int sc1, mn1, sc2, mn2;
  float d, dmin;
};

__device__ __forceinline__ ChunkScales chunk_scales(uint4 hdr, int c) {
  ChunkScales r;
  r.d = f16_bits_to_f32(hdr.x);
  r.dmin = f16_bits_to_f32(hdr.x >> 16);
  q4k_scale_min(hdr.y, hdr.z, hdr.w, 2 * c, r.sc1, r.mn1);
  q4k_scale_min(hdr.y, hdr.z, hdr.w, 2 * c + 1, r.sc2, r.mn2);
  r.d1 = r.d * (float)r.sc1;
  r.m1 = r.dmin * (float)r.mn1;
  r.d2 = r.d * (float)r.sc2;
  r.m2 = r.dmin * (float)r.mn2;
  return r;
}

// Exact small-integer -> f32 via the mantissa: 2^23 + v reinterpreted, minus 2^23.
__device__ __forceinline__ float u4_to_f32(uint32_t v) {
  return __int_as_float(0x4B000000 | v) - 8388608.0f;
}
// byte j (0..3) of v as an exact f32 (the same value as u4_to_f32 of that byte)
__device__ __forceinline__ float u8_to_f32(uint32_t v, int j) {
  return __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7440u | (uint32_t)j)) - 8388608.0f;
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void *p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// expf as the reference computes it.  Rust's f32::exp is glibc's expf, which
// since glibc 2.28 is Szabolcs Nagy's table-driven method (published in ARM's
// optimized-routines): in double precision, k = round(x * 32/ln2) and
// r = x * 32/ln2 - k, exp(x) = 2^(k/32) * P(r) with 2^(i/32) from a 32-entry
// table and P a cubic; the double result is rounded once to float.  On x86-64
// hosts with FMA (the ifunc variant glibc selects there) the reduction and
// the polynomial use fused multiply-adds, restated here with fma().  Checked
// against the host's expf on every float in [-104, 0] (the router's domain:
// logit - max), bit for bit.  The table holds 2^(i/32) rounded to nearest
// double; the three coefficients are the method's published values.
__device__ const uint64_t EXP2_I32[32] = {
    0x3ff0000000000000ull, 0x3ff059b0d3158574ull, 0x3ff0b5586cf9890full, 0x3ff11301d0125b51ull,
    0x3ff172b83c7d517bull, 0x3ff1d4873168b9aaull, 0x3ff2387a6e756238ull, 0x3ff29e9df51fdee1ull,
    0x3ff306fe0a31b715ull, 0x3ff371a7373aa9cbull, 0x3ff3dea64c123422ull, 0x3ff44e086061892dull,
    0x3ff4bfdad5362a27ull, 0x3ff5342b569d4f82ull, 0x3ff5ab07dd485429ull, 0x3ff6247eb03a5585ull,
    0x3ff6a09e667f3bcdull, 0x3ff71f75e8ec5f74ull, 0x3ff7a11473eb0187ull, 0x3ff82589994cce13ull,
    0x3ff8ace5422aa0dbull, 0x3ff93737b0cdc5e5ull, 0x3ff9c49182a3f090ull, 0x3ffa5503b23e255dull,
    0x3ffae89f995ad3adull, 0x3ffb7f76f2fb5e47ull, 0x3ffc199bdd85529cull, 0x3ffcb720dcef9069ull,
    0x3ffd5818dcfba487ull, 0x3ffdfc97337b9b5full, 0x3ffea4afa2a490daull, 0x3fff50765b6e4540ull};

// Branch-free, so unrolled calls overlap: the two out-of-range cases are
// selected at the end (the arithmetic on such x is discarded).
__device__ __forceinline__ float expf_ref(float x) {
  const double inv = 0x1.71547652b82fep+0 * 32.0, shift = 0x1.8p+52;
  const double c0 = 0x1.c6af84b912394p-5 / 32768.0, c1 = 0x1.ebfce50fac4f3p-3 / 1024.0,
               c2 = 0x1.62e42ff0c52d6p-1 / 32.0;
  const double xd = (double)x;
  double kd = __fma_rn(inv, xd, shift);             // round(x * 32/ln2) in the low bits
  const uint64_t ki = (uint64_t)__double_as_longlong(kd);
  kd -= shift;
  const double r = __fma_rn(inv, xd, -kd);          // |r| <= 1/2
  const uint32_t i = (uint32_t)(ki & 31u);
  // 2^(k/32) = 2^(i/32) * 2^((k - i)/32): add (k - i)/32 to the table entry's exponent
  const double s = __longlong_as_double((long long)(__ldg(&EXP2_I32[i]) + ((ki - i) << 47)));
  const double q = __fma_rn(c0, r, c1);
  const double r2 = __dmul_rn(r, r);
  double y = __fma_rn(c2, r, 1.0);
  y = __fma_rn(q, r2, y);
  const float res = __double2float_rn(__dmul_rn(y, s));
  return x < -0x1.9fe368p6f ? 0.0f                            // below log(2^-150): rounds to zero
         : x > 0x1.62e42ep6f ? __int_as_float(0x7f800000) : res;  // above log(2^128): overflow
}

// Programmatic dependent launch.  A kernel launched with launch_pdl may start
// while its predecessor in the stream is still running; pdl_wait blocks until
// that predecessor has completed and its writes are visible.  The kernels that
// use it read only constant data (weights) or data produced two or more
// launches back before pdl_wait, write nothing before it, and call
// pdl_launch_dependents only after it, so "two launches back" is always
// complete by the time a dependent starts.  Both are no-ops in a kernel
// launched normally.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// sigmoid of har-native-qwen35moe.rs:207-214, with the reference's exp
__device__ __forceinline__ float sigmoid_f(float v) {
  if (v >= 0.0f) return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf_ref(-v)));
  const float e = expf_ref(v);
  return __fdiv_rn(e, __fadd_rn(1.0f, e));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int WIDTH>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = WIDTH / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// sigmoid(gi . x) of one token row, computed by one warp: lane l accumulates
// the 4-value chunks l, l + 32, ... with fmaf (x, y, z, w in order), then the
// lanes are summed by a shuffle tree.  Every kernel that needs the shared
// expert's gate calls this, so a token's gate never depends on which kernel
// computed it or on the other tokens of the call.  x is 16-byte aligned, H a
// multiple of 4 (both checked by the callers).
__device__ __forceinline__ float shared_gate_warp(const float *gi, const float *x, int H, int lane) {
  float s = 0.0f;
  const float4 *x4 = reinterpret_cast<const float4 *>(x);
  if (((uintptr_t)gi & 15u) == 0) {
    const float4 *g4 = reinterpret_cast<const float4 *>(gi);
#pragma unroll 4
    for (int i = lane; i < H / 4; i += 32) {
      const float4 a = __ldg(g4 + i), b = x4[i];
      s = fmaf(a.x, b.x, s);
      s = fmaf(a.y, b.y, s);
      s = fmaf(a.z, b.z, s);
      s = fmaf(a.w, b.w, s);
    }
  } else {
    for (int i = lane; i < H / 4; i += 32) {
      const float4 b = x4[i];
      s = fmaf(__ldg(gi + 4 * i), b.x, s);
      s = fmaf(__ldg(gi + 4 * i + 1), b.y, s);
      s = fmaf(__ldg(gi + 4 * i + 2), b.z, s);
      s = fmaf(__ldg(gi + 4 * i + 3), b.w, s);
    }
  }
  return sigmoid_f(warp_sum(s));
}

}  // namespace har

// ---------------------------------------------------------------------------
// Host-side handle types (opaque in the C ABI).
// ---------------------------------------------------------------------------

struct har_cuda_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;      // stream kernels are launched on
  cudaStream_t own_stream = nullptr;  // the context's own stream
  int num_sms = 148;
  std::string last_error;
  int *d_status = nullptr;            // [0]: device error word (bit flags); [1]: the fused
                                      // router's completion counter (zero between calls)
  void *scratch = nullptr;            // grow-only scratch arena
  size_t scratch_bytes = 0;
  void *host_pinned = nullptr;        // pinned staging for *_host entry points
  size_t host_pinned_bytes = 0;
  void *io_dev = nullptr;             // device staging for *_host entry points
  size_t io_dev_bytes = 0;
  int64_t launches = 0;
  int tc_min_tokens = 0;              // tensor-core threshold override (0 = default)
  uint64_t epoch = 0;                 // bumped whenever scratch or staging is reallocated
  // CUDA graph of the last repeated har_cuda_moe_stack_host call (copies in,
  // the stack, copy out), replayed while the call's key is unchanged
  struct HostGraph {
    std::vector<uint64_t> layers;  // the layers' generation ids (never their addresses)
    int64_t T = 0;
    int32_t k = 0;
    uint32_t flags = 0;
    int tc_min = 0;
    uint64_t epoch = 0;
    cudaStream_t stream = nullptr;
    int seen = 0;  // consecutive calls with this key
    cudaGraphExec_t exec = nullptr;
  } host_graph;
  // opt-in per-launch CUDA-event profiling (har_cuda_profile_begin/end)
  bool prof_on = false;
  cudaEvent_t prof_pending = nullptr;
  struct ProfRec {
    const char *name;
    cudaEvent_t a, b;
  };
  std::vector<ProfRec> prof;
};

struct har_cuda_weights {
  const uint8_t *dev = nullptr;
  bool owned = false;
  int64_t E = 0, N = 0, K = 0;
  int32_t type = har::GGML_Q4_K;  // har::GGML_Q4_K or har::GGML_Q6_K
  int64_t row_bytes = 0;  // K/256 * (144 or 210)
  int64_t expert_bytes = 0;
  int device = 0;
};

// An encoded TMA tensor map (CUtensorMap: 128 bytes, 64-byte aligned).
struct alignas(64) TmaDesc {
  unsigned char bytes[128];
};

struct har_cuda_moe_layer {
  const har_cuda_weights *gate = nullptr, *up = nullptr, *down = nullptr;
  const har_cuda_weights *sh_gate = nullptr, *sh_up = nullptr, *sh_down = nullptr;
  const float *sh_gate_inp = nullptr;
  int64_t E = 0, H = 0, I = 0;
  // TMA maps of the weights for the tensor-core path: [E*rows][row_bytes]
  // bytes, box of 128 rows x one 144-byte super-block (tc_maps: encoded).
  bool tc_maps = false;
  TmaDesc map_gate, map_up, map_down, map_sh_gate, map_sh_up, map_sh_down;
  // A layer loaded from a GGUF file owns its tensors: the weights, and one
  // device buffer holding the f32 router [E][H] and shared-expert gate row.
  std::vector<har_cuda_weights *> owned;
  void *owned_dev = nullptr;
  const float *router = nullptr;  // ffn_gate_inp [E][H], or null
  // Process-unique id assigned at creation.  Caches key on it rather than on
  // the layer's address: a layer freed and another created at the same heap
  // address (with other weights) must not hit an entry of the first.
  uint64_t gen = 0;
};

namespace har {

// Error helpers shared by the .cu files.
int32_t set_error(har_cuda_ctx *ctx, int32_t code, const std::string &msg);
int32_t check_launch(har_cuda_ctx *ctx, const char *what);
// Call immediately before a kernel launch; check_launch closes the record.
void prof_begin(har_cuda_ctx *ctx);

// Launch with programmatic stream serialization (see pdl_wait).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}
int32_t ensure_scratch(har_cuda_ctx *ctx, size_t bytes);

// Kernel launchers (host functions defined in the kernel .cu files).
int32_t launch_q8k_quantize(har_cuda_ctx *ctx, const float *x, int64_t M, int64_t K,
                            uint8_t *out);
int32_t launch_gemv(har_cuda_ctx *ctx, const har_cuda_weights *w, int64_t expert,
                    const void *x, int act_kind, int64_t M, float *y);
int32_t launch_q3k_gemv(har_cuda_ctx *ctx, const har_cuda_weights *w, int64_t expert,
                        const float *x, int64_t M, float *y);
int32_t launch_q6k_gemv(har_cuda_ctx *ctx, const har_cuda_weights *w, int64_t expert,
                        const float *x, int64_t M, float *y);
int32_t launch_route_topk(har_cuda_ctx *ctx, const float *logits, int64_t T, int E, int k,
                          int32_t *ids, float *weights);
// gcnt: group_scratch_words(T * k, E) words of scratch (may be null for one CTA)
int32_t launch_group(har_cuda_ctx *ctx, const int32_t *ids, int64_t T, int k, int E,
                     int32_t *counts, int32_t *offsets, int32_t *order, int32_t *inv, int32_t *gcnt);
size_t group_scratch_words(int64_t n, int E);
int32_t launch_router_logits(har_cuda_ctx *ctx, const float *W, int E, int H, const float *x,
                             int64_t T, float *logits);
int32_t launch_route_fused(har_cuda_ctx *ctx, const float *W, int E, int H, const float *x,
                           int64_t T, int k, float *logits, int32_t *ids, float *weights,
                           bool *done);
int32_t run_moe_ffn(har_cuda_ctx *ctx, const har_cuda_moe_layer *layer, const float *x,
                    int64_t T, int k, const int32_t *ids, const float *weights, float *y,
                    uint32_t flags);
size_t moe_scratch_bytes(const har_cuda_ctx *ctx, const har_cuda_moe_layer *layer, int64_t T, int k,
                         uint32_t flags);
int32_t run_moe_ffn_in(har_cuda_ctx *ctx, const har_cuda_moe_layer *layer, const float *x,
                       int64_t T, int k, const int32_t *ids, const float *weights, float *y,
                       uint32_t flags, uint8_t *scratch);
// The same with the shared expert on tokens sh0 .. sh0 + shT - 1 only.
int32_t run_moe_ffn_range(har_cuda_ctx *ctx, const har_cuda_moe_layer *layer, const float *x,
                          int64_t T, int k, const int32_t *ids, const float *weights, float *y,
                          uint32_t flags, uint8_t *S, int64_t sh0, int64_t shT);
int32_t check_moe_args(har_cuda_ctx *ctx, const har_cuda_moe_layer *layer, int64_t T,
                       int32_t k, uint32_t flags);
// The decode path (HAR_CUDA_MOE_DECODE, k_moe_decode.cu) on a scratch region.
size_t moe_decode_scratch_bytes(const har_cuda_moe_layer *layer, int64_t T, int k);
int32_t run_moe_decode(har_cuda_ctx *ctx, const har_cuda_moe_layer *layer, const float *x,
                       int64_t T, int k, const int32_t *ids, const float *weights, float *y,
                       uint32_t flags, uint8_t *scratch);
int32_t encode_tmap_2d(har_cuda_ctx *ctx, TmaDesc *out, const void *base, int elem_bytes,
                       uint64_t rows, uint64_t cols, uint64_t row_stride, uint32_t box_rows,
                       uint32_t box_cols, bool swizzle128);
int32_t launch_gen_q4k(har_cuda_ctx *ctx, uint8_t *dst, int64_t rows, int64_t K,
                       uint64_t seed, int64_t row0, float mean, float stdv);

}  // namespace har
