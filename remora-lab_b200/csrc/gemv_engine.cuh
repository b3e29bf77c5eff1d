// gemv_engine.cuh — the CUDA-core Q4_K row-dot engine shared by the GEMV and
// MoE decode kernels.
//
// Work unit: a 64-value "chunk" = 32 bytes of nibbles of one super-block plus
// that block's 16-byte header (d, dmin, 12 scale bytes).  Chunk c of block b
// covers values 64c..64c+63: low nibbles are sub-block 2c, high nibbles
// sub-block 2c+1 (q4k_dot's loop, har/crates/har-demo/src/bin/har-native-qwen3.rs:157-168).
// A row of K values has C = K/64 chunks; LPR = min(32, C) lanes share a row
// and each lane owns CPL = ceil(C/32) fixed chunk positions, so its slice of
// the activations is loaded into registers once and reused for every row the
// warp visits.  Rows are read with 128-bit loads straight from HBM.
//
// Two activation kinds:
//   ACT_F32 — f32 activations; per sub-block sum_q q*x is accumulated with
//             FMAs and combined as d1*sum(q*x) - m1*sum(x) (the f32 value
//             (d1*q - m1)*x of q4k_dot, reassociated; tolerance-checked).
//   ACT_Q8K — Q8_K activations; per sub-block integer dot products with
//             __dp4a, combined as (d*dx)*I1 - (dmin*dx)*I2 per chunk.
#pragma once

#include "har_internal.cuh"

namespace har {

enum : int { ACT_F32 = 0, ACT_Q8K = 1 };

// Shared-memory image of MT tokens' activations for one K.
//  F32: xs[t][K] f32, sums[t][2*C] f32 (per-sub-block sums of x)
//  Q8K: qs[t][K] int8, dx[t][K/256] f32, bsum[t][2*C] int (per-sub-block bsums)
template <int ACT>
struct ActSmem;

template <>
struct ActSmem<ACT_F32> {
  static __host__ __device__ size_t bytes(int MT, int K) {
    return (size_t)MT * K * 4 + (size_t)MT * (K / 32) * 4;
  }
};
template <>
struct ActSmem<ACT_Q8K> {
  static __host__ __device__ size_t bytes(int MT, int K) {
    return (size_t)MT * K + (size_t)MT * (K / 256) * 4 + (size_t)MT * (K / 32) * 4;
  }
};

// Per-32-value sub-block sums of MT f32 rows already in shared memory
// (xs[t][K] at the start of smem); ends with a CTA barrier.
__device__ __forceinline__ void stage_f32_sums(uint8_t *smem, int MT, int K) {
  const float *xs = reinterpret_cast<const float *>(smem);
  float *sums = reinterpret_cast<float *>(smem) + (size_t)MT * K;
  const int nsub = K / 32;
  for (int i = threadIdx.x; i < MT * nsub; i += blockDim.x) {
    const int t = i / nsub, s = i - t * nsub;
    const float *p = xs + (size_t)t * K + 32 * s;
    float acc = 0.0f;
#pragma unroll 8
    for (int j = 0; j < 32; ++j) acc += p[j];
    sums[(size_t)t * nsub + s] = acc;
  }
  __syncthreads();
}

// Stage f32 activation rows (row pointers may be null for padding tokens).
__device__ __forceinline__ void stage_f32(uint8_t *smem, const float *const *rows, int MT, int K) {
  float *xs = reinterpret_cast<float *>(smem);
  const int nvec = K / 4;
  for (int i = threadIdx.x; i < MT * nvec; i += blockDim.x) {
    const int t = i / nvec, v = i - t * nvec;
    float4 val = rows[t] ? reinterpret_cast<const float4 *>(rows[t])[v] : make_float4(0, 0, 0, 0);
    reinterpret_cast<float4 *>(xs + (size_t)t * K)[v] = val;
  }
  __syncthreads();
  stage_f32_sums(smem, MT, K);
}

// Stage packed Q8_K activation rows (292-byte blocks).
__device__ __forceinline__ void stage_q8k(uint8_t *smem, const uint8_t *const *rows, int MT, int K) {
  int8_t *qs = reinterpret_cast<int8_t *>(smem);
  float *dx = reinterpret_cast<float *>(smem + (size_t)MT * K);
  int *bsum = reinterpret_cast<int *>(dx + (size_t)MT * (K / 256));
  const int nb = K / 256;
  // qs: 64 words per block
  for (int i = threadIdx.x; i < MT * nb * 64; i += blockDim.x) {
    const int t = i / (nb * 64), r = i - t * nb * 64, b = r >> 6, w = r & 63;
    uint32_t v = rows[t] ? reinterpret_cast<const uint32_t *>(rows[t] + (size_t)b * Q8K_BYTES + 4)[w] : 0u;
    reinterpret_cast<uint32_t *>(qs + (size_t)t * K + 256 * b)[w] = v;
  }
  for (int i = threadIdx.x; i < MT * nb; i += blockDim.x) {
    const int t = i / nb, b = i - t * nb;
    dx[(size_t)t * nb + b] = rows[t] ? *reinterpret_cast<const float *>(rows[t] + (size_t)b * Q8K_BYTES) : 0.0f;
  }
  // per 32-value sub-block: bsums[2s] + bsums[2s+1]
  for (int i = threadIdx.x; i < MT * nb * 8; i += blockDim.x) {
    const int t = i / (nb * 8), r = i - t * nb * 8, b = r >> 3, s = r & 7;
    int v = 0;
    if (rows[t]) {
      const int16_t *bs = reinterpret_cast<const int16_t *>(rows[t] + (size_t)b * Q8K_BYTES + 260);
      v = (int)bs[2 * s] + (int)bs[2 * s + 1];
    }
    bsum[(size_t)t * (K / 32) + 8 * b + s] = v;
  }
  __syncthreads();
}

// 16-byte load from shared memory by its shared-window address: explicit, so
// a staged row is never read through the generic path.  Volatile keeps it
// after the barrier wait that publishes the row.
__device__ __forceinline__ uint4 lds_u4(uint32_t saddr) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "r"(saddr));
  return r;
}
__device__ __forceinline__ float4 lds_f4(uint32_t saddr) {
  const uint4 r = lds_u4(saddr);
  return make_float4(__uint_as_float(r.x), __uint_as_float(r.y), __uint_as_float(r.z), __uint_as_float(r.w));
}

// Per-lane activation registers for one chunk of one token.
template <int ACT>
struct LaneAct;

template <>
struct LaneAct<ACT_F32> {
  float lo[32], hi[32];
  float slo, shi;
  __device__ __forceinline__ void load(const uint8_t *smem, int MT, int K, int t, int chunk) {
    const float *xs = reinterpret_cast<const float *>(smem) + (size_t)t * K + 64 * chunk;
    const float *sums = reinterpret_cast<const float *>(smem) + (size_t)MT * K + (size_t)t * (K / 32);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float4 a = reinterpret_cast<const float4 *>(xs)[i];
      float4 b = reinterpret_cast<const float4 *>(xs + 32)[i];
      lo[4 * i] = a.x; lo[4 * i + 1] = a.y; lo[4 * i + 2] = a.z; lo[4 * i + 3] = a.w;
      hi[4 * i] = b.x; hi[4 * i + 1] = b.y; hi[4 * i + 2] = b.z; hi[4 * i + 3] = b.w;
    }
    slo = sums[2 * chunk];
    shi = sums[2 * chunk + 1];
  }
  // The chunk from a plain f32 row in shared memory (64 floats at src,
  // 16-byte aligned), with the two sub-block sums taken in registers: a fixed
  // pairwise tree, so the sums do not depend on the launch shape.
  __device__ __forceinline__ void load_row(const float *src) {
    const uint32_t sa = (uint32_t)__cvta_generic_to_shared(src);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 a = lds_f4(sa + 16 * i), b = lds_f4(sa + 128 + 16 * i);
      lo[4 * i] = a.x; lo[4 * i + 1] = a.y; lo[4 * i + 2] = a.z; lo[4 * i + 3] = a.w;
      hi[4 * i] = b.x; hi[4 * i + 1] = b.y; hi[4 * i + 2] = b.z; hi[4 * i + 3] = b.w;
    }
    slo = tree_sum32(lo);
    shi = tree_sum32(hi);
  }
  static __device__ __forceinline__ float tree_sum32(const float (&v)[32]) {
    float t[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) t[i] = v[i] + v[i + 16];
#pragma unroll
    for (int i = 0; i < 8; ++i) t[i] += t[i + 8];
#pragma unroll
    for (int i = 0; i < 4; ++i) t[i] += t[i + 4];
    return (t[0] + t[2]) + (t[1] + t[3]);
  }
};

template <>
struct LaneAct<ACT_Q8K> {
  int lo[8], hi[8];
  int blo, bhi;
  float dx;
  __device__ __forceinline__ void load(const uint8_t *smem, int MT, int K, int t, int chunk) {
    const int8_t *qs = reinterpret_cast<const int8_t *>(smem) + (size_t)t * K + 64 * chunk;
    const float *dxs = reinterpret_cast<const float *>(smem + (size_t)MT * K);
    const int *bsum = reinterpret_cast<const int *>(dxs + (size_t)MT * (K / 256));
    uint4 a0 = reinterpret_cast<const uint4 *>(qs)[0], a1 = reinterpret_cast<const uint4 *>(qs)[1];
    uint4 b0 = reinterpret_cast<const uint4 *>(qs)[2], b1 = reinterpret_cast<const uint4 *>(qs)[3];
    lo[0] = a0.x; lo[1] = a0.y; lo[2] = a0.z; lo[3] = a0.w;
    lo[4] = a1.x; lo[5] = a1.y; lo[6] = a1.z; lo[7] = a1.w;
    hi[0] = b0.x; hi[1] = b0.y; hi[2] = b0.z; hi[3] = b0.w;
    hi[4] = b1.x; hi[5] = b1.y; hi[6] = b1.z; hi[7] = b1.w;
    dx = dxs[(size_t)t * (K / 256) + chunk / 4];
    blo = bsum[(size_t)t * (K / 32) + 2 * chunk];
    bhi = bsum[(size_t)t * (K / 32) + 2 * chunk + 1];
  }
};

// Raw weight chunk held in registers.
struct WChunk {
  uint4 hdr, q0, q1;
};

__device__ __forceinline__ WChunk load_wchunk(const uint8_t *row, int chunk) {
  const uint8_t *blk = row + (size_t)(chunk >> 2) * Q4K_BYTES;
  const int c = chunk & 3;
  WChunk w;
  w.hdr = __ldg(reinterpret_cast<const uint4 *>(blk));
  w.q0 = __ldg(reinterpret_cast<const uint4 *>(blk + 16 + 32 * c));
  w.q1 = __ldg(reinterpret_cast<const uint4 *>(blk + 32 + 32 * c));
  return w;
}

// The same chunk from a row staged in shared memory (plain loads: the
// read-only global path must not see a shared address).
__device__ __forceinline__ WChunk load_wchunk_s(const uint8_t *row, int chunk) {
  const uint32_t blk = (uint32_t)__cvta_generic_to_shared(row) + (uint32_t)(chunk >> 2) * Q4K_BYTES;
  const uint32_t c = (uint32_t)(chunk & 3);
  WChunk w;
  w.hdr = lds_u4(blk);
  w.q0 = lds_u4(blk + 16 + 32 * c);
  w.q1 = lds_u4(blk + 32 + 32 * c);
  return w;
}

__device__ __forceinline__ float chunk_dot(const WChunk &w, int chunk, const LaneAct<ACT_Q8K> &a) {
  const uint32_t q[8] = {w.q0.x, w.q0.y, w.q0.z, w.q0.w, w.q1.x, w.q1.y, w.q1.z, w.q1.w};
  int slo = 0, shi = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    slo = __dp4a((int)(q[i] & 0x0F0F0F0Fu), a.lo[i], slo);
    shi = __dp4a((int)((q[i] >> 4) & 0x0F0F0F0Fu), a.hi[i], shi);
  }
  int sc1, m1, sc2, m2;
  const int c = chunk & 3;
  q4k_scale_min(w.hdr.y, w.hdr.z, w.hdr.w, 2 * c, sc1, m1);
  q4k_scale_min(w.hdr.y, w.hdr.z, w.hdr.w, 2 * c + 1, sc2, m2);
  const float d = f16_bits_to_f32(w.hdr.x), dmin = f16_bits_to_f32(w.hdr.x >> 16);
  const int i1 = sc1 * slo + sc2 * shi;
  const int i2 = m1 * a.blo + m2 * a.bhi;
  return (d * a.dx) * (float)i1 - (dmin * a.dx) * (float)i2;
}

// The f32 chunk dot: sum_q q*x per sub-block, then d1*sum(q*x) - m1*sum(x)
// (q4k_dot's per-value (d1*q - m1)*x, reassociated; tolerance-checked).  Each
// nibble becomes an exact f32 by a byte permute into the mantissa of 2^23 and
// a subtraction of 2^23; values go through Blackwell's packed f32x2 add and
// FMA two at a time, into four accumulators per sub-block (bytes 0-1 and 2-3
// of each word as two pairs), added pairwise at the end.  Two instructions per
// value instead of three, and a dependent FMA depth of 8: the decode GEMVs and
// kernels are bound by instruction issue and latency.
__device__ __forceinline__ float2 u8x2_to_f32(uint32_t v, int j) {
  const float2 b = make_float2(__uint_as_float(__byte_perm(v, 0x4B000000u, 0x7440u | (uint32_t)j)),
                               __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7440u | (uint32_t)(j + 1))));
  return __fadd2_rn(b, make_float2(-8388608.0f, -8388608.0f));
}
__device__ __forceinline__ float chunk_dot(const WChunk &w, int chunk, const LaneAct<ACT_F32> &a) {
  const uint32_t q[8] = {w.q0.x, w.q0.y, w.q0.z, w.q0.w, w.q1.x, w.q1.y, w.q1.z, w.q1.w};
  float2 l01 = make_float2(0.0f, 0.0f), l23 = l01, h01 = l01, h23 = l01;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t lo = q[i] & 0x0F0F0F0Fu, hi = (q[i] >> 4) & 0x0F0F0F0Fu;
    l01 = __ffma2_rn(u8x2_to_f32(lo, 0), make_float2(a.lo[4 * i], a.lo[4 * i + 1]), l01);
    l23 = __ffma2_rn(u8x2_to_f32(lo, 2), make_float2(a.lo[4 * i + 2], a.lo[4 * i + 3]), l23);
    h01 = __ffma2_rn(u8x2_to_f32(hi, 0), make_float2(a.hi[4 * i], a.hi[4 * i + 1]), h01);
    h23 = __ffma2_rn(u8x2_to_f32(hi, 2), make_float2(a.hi[4 * i + 2], a.hi[4 * i + 3]), h23);
  }
  const float sl = (l01.x + l01.y) + (l23.x + l23.y), sh = (h01.x + h01.y) + (h23.x + h23.y);
  const ChunkScales s = chunk_scales(w.hdr, chunk & 3);
  return (s.d1 * sl - s.m1 * a.slo) + (s.d2 * sh - s.m2 * a.shi);
}

// The decode kernels' name for the same dot.
__device__ __forceinline__ float chunk_dot_ilp(const WChunk &w, int chunk, const LaneAct<ACT_F32> &a) {
  return chunk_dot(w, chunk, a);
}

// Lanes per row, chunks per lane and tokens per pass for a given K.
struct GemvShape {
  int C;    // chunks per row
  int LPR;  // lanes per row
  int CPL;  // chunks per lane
  int RPW;  // rows per warp iteration (32 / LPR)
};

__host__ __device__ inline GemvShape gemv_shape(int K) {
  GemvShape s;
  s.C = K / 64;
  if (s.C >= 32) {
    s.LPR = 32;
    s.CPL = (s.C + 31) / 32;
  } else {
    int l = 1;
    while (l < s.C) l <<= 1;  // next power of two >= C
    s.LPR = l;
    s.CPL = 1;
  }
  s.RPW = 32 / s.LPR;
  return s;
}

template <int LPR>
__device__ __forceinline__ float lane_group_sum(float v) {
  return group_sum<LPR>(v);
}

}  // namespace har
