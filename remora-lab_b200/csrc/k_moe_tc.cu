// k_moe_tc.cu — the tensor-core path of the expert FFN: grouped per-expert
// gate/up GEMM with fused SwiGLU, and the down GEMM, on tcgen05 for experts
// whose token count reaches a threshold (the rest take the CUDA-core GEMV path
// in k_moe.cu).  Semantics are compose_moe_route's
// (har/crates/har-demo/src/bin/har-native-qwen35moe.rs:979-1048) per token.
//
// Shape: the weights are the MMA's M side ("swap AB"): a tile is 128 weight
// rows x up to 64 token columns, so a tile of W is dequantised once for up to
// 64 tokens.  D = W_tile * X^T accumulates in TMEM (f32).
//   gate/up: two accumulators (gate rows and up rows of the same 128
//            intermediate indices); epilogue a = silu(g) * u -> a16[slot][i] (f16).
//   down:    one accumulator; epilogue ybuf[slot][h] (f32), then the common
//            combine kernel applies the routing weights in slot order.
//
// With few tokens per expert the MMAs are narrow (N = 16..64) and a single
// issuing warp cannot keep up with HBM: each tcgen05.mma costs the issuer
// about 100 cycles whatever N is, i.e. ~20 weights per cycle, while one SM's
// share of HBM bandwidth is ~40 Q4_K weights per cycle.  So two warps issue,
// each for alternate 64-value K-steps into its own accumulator set, and the
// epilogue adds the two partial sums.
//
// One persistent CTA per SM, warp-specialised, every handoff an mbarrier:
//   TMA threads:  one loads raw Q4_K boxes (128 rows x one 144-byte
//                 super-block per matrix) into a raw ring in shared memory;
//                 another loads 128-byte-swizzled f16 token tiles (64 values x
//                 16/32/64 rows: the smallest box covering the tile's tokens,
//                 which sit in slot order) into a B ring whose 16 KB slots
//                 hold 128/box-rows K-steps each.
//   dequant warps: two teams of four, team t taking the K-steps of issuer t,
//                 turn the raw blocks into f16 weights with packed-f16
//                 arithmetic and store them straight into the team's two
//                 tensor-memory stages with tcgen05.st (warp w owns TMEM lanes
//                 32*(w%4).. = those rows).  Keeping the weight operand out of
//                 shared memory keeps its write and its tensor-core read off
//                 the shared-memory bandwidth.
//   MMA warps:    4 x tcgen05.mma (K=16, A from TMEM, B from shared memory)
//                 per matrix per K-step; tcgen05.commit frees the weight stage
//                 and the B slot, and signals the epilogue at the end of a tile.
//   epilogue warps: tcgen05.ld both partial accumulators, add, apply the
//                 epilogue, store, then free the accumulator columns.
// No multicast: every TMA load reads this GPU's memory into this CTA only.
// Operands are f16 (same tensor rate as bf16, 3 more mantissa bits): each
// weight is d*(sc*q) with sc*q exact, minus dmin*m rounded to f16, rounded
// once more to f16; each activation is rounded once to f16; accumulation is f32.
#include <algorithm>

#include "gemv_engine.cuh"
#include "moe_tc.cuh"
#include "tc_ptx.cuh"

namespace har {

// Shared-memory plan: raw ring (one super-block step = 4 K-steps per slot)
// and B ring (16 KB slots of 128/box-rows K-steps).  The f16 weight operand
// does not touch shared memory: it is written to tensor memory.
template <int NA>
struct TcSmem {
  static constexpr int RAW_SLOTS = NA == 2 ? 4 : 6;
  static constexpr int B_SLOTS = 4;
  static constexpr int BSL = 128 * 128;           // 16 KB: 128 rows of 64 f16
  static constexpr int RAWSL = NA * TC_M * Q4K_BYTES;
  static constexpr int OFF_B = 0;                 // 1024-aligned swizzled buffers first
  static constexpr int OFF_RAW = OFF_B + B_SLOTS * BSL;
  static constexpr int BYTES = OFF_RAW + RAW_SLOTS * RAWSL;
};

// Tensor-memory plan (512 columns x 128 lanes): accumulators in 64-column
// quarters at [0, A_COL0), then TC_ISSUERS x 2 f16 weight stages of NA x 32
// columns (one 64-value K-step: row = lane, two f16 per column in K order).
// A tile with token box rows_b takes ceil(TC_ISSUERS * NA * rows_b / 64)
// quarters: issuer i's accumulator of matrix m sits at column
// (i * NA + m) * rows_b of the tile's first quarter.
template <int NA>
struct TcTmem {
  static constexpr int A_STAGES = 2 * TC_ISSUERS;
  static constexpr int A_COL0 = TC_TMEM_COLS - A_STAGES * NA * 32;
  static constexpr int NQ = A_COL0 / 64;
  static __device__ __forceinline__ int quarters(int rows_b) {
    return (TC_ISSUERS * NA * rows_b + 63) / 64;
  }
};

// Smallest token-tile box (16, 32 or 64 rows) covering n tokens.
__device__ __forceinline__ int tc_box(int n) { return n <= 16 ? 0 : n <= 32 ? 1 : 2; }

// Map a token-tile index to (expert, or E for the shared expert; token
// count; first slot).  Routed tiles come from the grouping kernel's table,
// the shared expert's tiles follow them.  False when the index is past the work.
__device__ __forceinline__ bool tc_tile(const TcParams &p, int routed_tt, int ttg, int &e,
                                        int &ntok, int &slot0) {
  if (ttg < routed_tt) {
    const int2 v = p.tt_info[ttg];
    e = v.x & 0xffff;
    ntok = v.x >> 16;
    slot0 = v.y;
    return true;
  }
  if (!p.shared_tc) return false;
  const int t0 = (ttg - routed_tt) * TC_NT;
  e = p.E;
  ntok = min(TC_NT, p.T - t0);
  slot0 = p.n + t0;
  return ntok > 0;
}

// Accumulator quarters of the next tile: `qc` is the ring cursor (the MMA
// warps and the epilogue walk the same tiles, so they agree); a tile that does
// not fit before the end wraps to quarter 0.  Returns the first quarter.
template <int NA>
__device__ __forceinline__ int tc_take_quarters(int &qc, int nq) {
  if (qc + nq > TcTmem<NA>::NQ) qc = 0;
  const int q0 = qc;
  qc += nq;
  if (qc == TcTmem<NA>::NQ) qc = 0;
  return q0;
}

// Dequantise one 32-value sub-block of a raw Q4_K block in shared memory
// (`blk` = the 144-byte block; chunk c of 4; `hi` selects the high nibbles,
// i.e. the odd sub-block) into 16 f16x2 words in K order.
// Packed f16 arithmetic, two values per instruction:
//   byte-permute each nibble q into the f16 bit pattern 0x64qq = 1024 + q,
//   hfma2((1024 + q), sc, -1024*sc) = sc*q exactly (an integer <= 945),
//   hfma2(sc*q, d, -(dmin*m)) = d*sc*q - dmin*m rounded once to f16
// (d is the block's f16 scale, exact; dmin*m is rounded to f16 first).
__device__ __forceinline__ void tc_dequant_sub(const uint8_t *blk, int c, int hi, uint32_t *o) {
  const uint4 hdr = *reinterpret_cast<const uint4 *>(blk);
  const uint4 q0 = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * c);
  const uint4 q1 = *reinterpret_cast<const uint4 *>(blk + 32 + 32 * c);
  int sc, mn;
  q4k_scale_min(hdr.y, hdr.z, hdr.w, 2 * c + hi, sc, mn);
  const __half2 d2 = __half2half2(__ushort_as_half((unsigned short)(hdr.x & 0xffffu)));
  const __half2 sc2 = __half2half2(__int2half_rn(sc));
  const __half2 nsc2 = __half2half2(__int2half_rn(-1024 * sc));
  const float dmin = f16_bits_to_f32(hdr.x >> 16);
  const __half2 c2 = __half2half2(__float2half_rn(-(dmin * (float)mn)));
  const uint32_t q[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {  // word i holds values 4i .. 4i+3 of the sub-block
    const uint32_t v = hi ? (q[i] >> 4) & 0x0F0F0F0Fu : q[i] & 0x0F0F0F0Fu;
    const uint32_t p01 = __byte_perm(v, 0x64646464u, 0x5140);  // (1024+q0, 1024+q1)
    const uint32_t p23 = __byte_perm(v, 0x64646464u, 0x7362);  // (1024+q2, 1024+q3)
    const __half2 s01 = __hfma2(*reinterpret_cast<const __half2 *>(&p01), sc2, nsc2);
    const __half2 s23 = __hfma2(*reinterpret_cast<const __half2 *>(&p23), sc2, nsc2);
    const __half2 w01 = __hfma2(s01, d2, c2);
    const __half2 w23 = __hfma2(s23, d2, c2);
    o[2 * i] = *reinterpret_cast<const uint32_t *>(&w01);
    o[2 * i + 1] = *reinterpret_cast<const uint32_t *>(&w23);
  }
}

__device__ __forceinline__ float tc_silu(float v) { return v / (1.0f + expf(-v)); }

// Bounded wait shared by the roles: false (and the CTA-wide abort flag set)
// when the barrier phase did not complete within TC_WAIT_LIMIT polls.
__device__ __forceinline__ bool tc_wait(uint64_t *bar, uint32_t parity, volatile int *abort_s) {
  if (*abort_s) return false;
  if (tc::mbar_wait(bar, parity, TC_WAIT_LIMIT)) return true;
  *abort_s = 1;
  return false;
}
// The same for a whole warp: lane 0 polls, the outcome is broadcast, and the
// warp leaves converged (the warp-wide MMA forms need it so).
__device__ __forceinline__ bool tc_wait_warp(uint64_t *bar, uint32_t parity, volatile int *abort_s,
                                             int lane) {
  bool ok = true;
  if (lane == 0) ok = tc_wait(bar, parity, abort_s);
  return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
}

// NA = number of A matrices (2: gate and up with SwiGLU epilogue; 1: down).
template <int NA>
__global__ void __launch_bounds__(TC_THREADS, 1) moe_tc_kernel(const __grid_constant__ TcMaps maps,
                                                               const TcParams p) {
  using L = TcSmem<NA>;
  using TM = TcTmem<NA>;
  extern __shared__ uint8_t tc_raw[];
  constexpr int RS = L::RAW_SLOTS, BS = L::B_SLOTS, AS = TM::A_STAGES, NQ = TM::NQ;
  __shared__ uint64_t bars[2 * RS + 2 * BS + 2 * AS + 2 * NQ];
  uint64_t *raw_full = bars, *raw_empty = bars + RS, *b_full = bars + 2 * RS, *b_empty = bars + 2 * RS + BS;
  uint64_t *a_full = bars + 2 * RS + 2 * BS, *a_empty = a_full + AS;
  uint64_t *acc_full = a_empty + AS, *acc_empty = acc_full + NQ;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  volatile int *abort_s = &abort_flag;
  uint8_t *sm = tc_raw + ((1024u - (tc::smem_u32(tc_raw) & 1023u)) & 1023u);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (warp == 0) {
    tc::tmem_alloc(&tmem_base, TC_TMEM_COLS);
    tc::tmem_relinquish();
  }
  if (tid == 32) {
    for (int s = 0; s < RS; ++s) {
      tc::mbar_init(raw_full + s, 1);
      tc::mbar_init(raw_empty + s, TC_DQ_WARPS);
    }
    for (int s = 0; s < AS; ++s) {
      tc::mbar_init(a_full + s, TC_DQ_WARPS / TC_ISSUERS);  // one team fills a stage
      tc::mbar_init(a_empty + s, 1);
    }
    for (int q = 0; q < NQ; ++q) {
      tc::mbar_init(acc_full + q, TC_ISSUERS);
      tc::mbar_init(acc_empty + q, 4);
    }
    for (int s = 0; s < BS; ++s) {
      tc::mbar_init(b_full + s, 1);
      tc::mbar_init(b_empty + s, TC_ISSUERS);
    }
    tc::fence_mbar_init();
    abort_flag = 0;
  }
  if (tid == 0) {
    tc::tma_prefetch_desc(&maps.a0);
    tc::tma_prefetch_desc(&maps.b[0]);
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = tmem_base;

  const int RT = p.rows / TC_M;
  const int KSTEPS = p.K / 64, KSB = p.K / 256;
  const int routed_tt = *p.n_tt;
  const int total_tt = routed_tt + (p.shared_tc ? (p.T + TC_NT - 1) / TC_NT : 0);
  const int total = total_tt * RT;

  if (warp == TC_WARP_TMA) {
    // ---------------- producer: raw weight boxes ----------------
    if (lane == 0) {
      uint32_t raw_it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
        int e, ntok, slot0;
        if (!tc_tile(p, routed_tt, tile / RT, e, ntok, slot0)) continue;
        const int r0 = (tile % RT) * TC_M;
        const bool sh = e == p.E;
        const void *m0 = sh ? (const void *)&maps.sh0 : (const void *)&maps.a0;
        const void *m1 = sh ? (const void *)&maps.sh1 : (const void *)&maps.a1;
        const int ya = sh ? r0 : e * p.rows + r0;
        for (int s = 0; ok && s < KSB; ++s) {
          const int rs = raw_it % RS;
          if (!(ok = tc_wait(raw_empty + rs, ((raw_it / RS) & 1u) ^ 1u, abort_s))) break;
          tc::mbar_expect_tx(raw_full + rs, (uint32_t)L::RAWSL);
          uint8_t *dst = sm + L::OFF_RAW + rs * L::RAWSL;
          tc::tma_load_2d(dst, m0, s * Q4K_BYTES, ya, raw_full + rs);
          if (NA == 2) tc::tma_load_2d(dst + TC_M * Q4K_BYTES, m1, s * Q4K_BYTES, ya, raw_full + rs);
          ++raw_it;
        }
      }
    }
  } else if (warp == TC_WARP_BTMA) {
    // ---------------- producer: token tiles (box sized to the tile) ----------------
    if (lane == 0) {
      uint32_t b_it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
        int e, ntok, slot0;
        if (!tc_tile(p, routed_tt, tile / RT, e, ntok, slot0)) continue;
        const int bx = tc_box(ntok);
        const void *bm = &maps.b[bx];
        const int rows_b = 16 << bx, kpb = 128 / rows_b;  // K-steps per B slot
        const uint32_t sub_bytes = (uint32_t)rows_b * 128u;
        for (int s0 = 0; ok && s0 < KSTEPS; s0 += kpb) {
          const int bs = b_it % BS, nsub = min(kpb, KSTEPS - s0);
          if (!(ok = tc_wait(b_empty + bs, ((b_it / BS) & 1u) ^ 1u, abort_s))) break;
          tc::mbar_expect_tx(b_full + bs, sub_bytes * (uint32_t)nsub);
          for (int j = 0; j < nsub; ++j)
            tc::tma_load_2d(sm + L::OFF_B + bs * L::BSL + j * sub_bytes, bm, (s0 + j) * 64, slot0, b_full + bs);
          ++b_it;
        }
      }
    }
  } else if (warp == TC_WARP_MMA0 || warp == TC_WARP_MMA1) {
    // ---------------- MMA issuers (whole warp, one elected lane issues) ----------------
    const int is = warp == TC_WARP_MMA0 ? 0 : 1;  // this warp takes K-steps ks % 2 == is
    uint32_t j = 0, b_it = 0, par = 0;  // par bit q: parity of quarter q's uses
    int qc = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
      int e, ntok, slot0;
      if (!tc_tile(p, routed_tt, tile / RT, e, ntok, slot0)) continue;
      const int rows_b = 16 << tc_box(ntok), kpb = 128 / rows_b, nq = TM::quarters(rows_b);
      const int q0 = tc_take_quarters<NA>(qc, nq);
      for (int u = 0; ok && u < nq; ++u)
        ok = tc_wait_warp(acc_empty + q0 + u, ((par >> (q0 + u)) & 1u) ^ 1u, abort_s, lane);
      if (!ok) break;
      tc::tc_fence_after();
      const uint32_t idesc = tc::idesc_f16(TC_M, (ntok + 15) & ~15);
      const uint32_t dcol = tmem + (uint32_t)(q0 * 64 + is * NA * rows_b);
      for (int ks = is; ks < KSTEPS; ks += 2, ++j) {
        const int st = is * 2 + (int)(j & 1u);
        if (!(ok = tc_wait_warp(a_full + st, (j >> 1) & 1u, abort_s, lane))) break;
        const int s0 = ks - ks % kpb, send = min(s0 + kpb, KSTEPS), bs = b_it % BS;
        if (ks == s0 + is)
          if (!(ok = tc_wait_warp(b_full + bs, (b_it / BS) & 1u, abort_s, lane))) break;
        tc::tc_fence_after();
        const uint64_t bdesc0 =
            tc::desc_sw128(tc::smem_u32(sm + L::OFF_B + bs * L::BSL) + (uint32_t)((ks - s0) * rows_b * 128));
        const uint32_t acol = tmem + (uint32_t)(TM::A_COL0 + st * NA * 32);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
          for (int m = 0; m < NA; ++m)
            tc::mma_f16_ts_w(dcol + (uint32_t)(m * rows_b), acol + (uint32_t)(m * 32 + kk * 8),
                             bdesc0 + (uint64_t)(2 * kk), idesc, (ks >= 2 || kk > 0) ? 1u : 0u);
        }
        tc::mma_commit_w(a_empty + st);
        if (ks == send - 2 + is) {
          tc::mma_commit_w(b_empty + bs);
          ++b_it;
        }
      }
      if (!ok) break;
      for (int u = 0; u < nq; ++u) tc::mma_commit_w(acc_full + q0 + u);
      par ^= ((1u << nq) - 1u) << q0;
    }
  } else if (warp < TC_WARP_DQ0) {
    // ---------------- epilogue: TMEM -> global ----------------
    const int g = warp & 3;  // TMEM lane group this warp may access
    const uint32_t lane_addr = (uint32_t)(32 * g) << 16;
    uint32_t par = 0;
    int qc = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
      int e, ntok, slot0;
      if (!tc_tile(p, routed_tt, tile / RT, e, ntok, slot0)) continue;
      const int rows_b = 16 << tc_box(ntok), nq = TM::quarters(rows_b);
      const int q0 = tc_take_quarters<NA>(qc, nq);
      for (int u = 0; ok && u < nq; ++u)
        ok = tc_wait_warp(acc_full + q0 + u, (par >> (q0 + u)) & 1u, abort_s, lane);
      if (!ok) break;
      tc::tc_fence_after();
      const int row = (tile % RT) * TC_M + 32 * g + lane;
      const uint32_t dcol = tmem + lane_addr + (uint32_t)(q0 * 64);
      for (int col = 0; col < ntok; col += 16) {
        uint32_t g0[16], g1[16];
        tc::tmem_ld16(dcol + (uint32_t)col, g0);                         // issuer 0, matrix 0
        tc::tmem_ld16(dcol + (uint32_t)(NA * rows_b + col), g1);          // issuer 1, matrix 0
        if (NA == 2) {
          uint32_t u0[16], u1[16];
          tc::tmem_ld16(dcol + (uint32_t)(rows_b + col), u0);             // issuer 0, matrix 1
          tc::tmem_ld16(dcol + (uint32_t)(3 * rows_b + col), u1);         // issuer 1, matrix 1
          tc::tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 16; ++c)
            if (col + c < ntok) {
              const float gv = __uint_as_float(g0[c]) + __uint_as_float(g1[c]);
              const float uv = __uint_as_float(u0[c]) + __uint_as_float(u1[c]);
              p.a16[((int64_t)slot0 + col + c) * p.out_ld + row] = __float2half_rn(__fmul_rn(tc_silu(gv), uv));
            }
        } else {
          tc::tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 16; ++c)
            if (col + c < ntok)
              p.ybuf[((int64_t)slot0 + col + c) * p.out_ld + row] = __uint_as_float(g0[c]) + __uint_as_float(g1[c]);
        }
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0)
        for (int u = 0; u < nq; ++u) tc::mbar_arrive(acc_empty + q0 + u);
      par ^= ((1u << nq) - 1u) << q0;
    }
  } else {
    // ---------------- dequantisers: raw Q4_K -> f16 weight stages in TMEM ----------------
    // Team t (four warps) takes the K-steps of issuer t, filling that issuer's
    // two stages in turn.  Warp w may store only TMEM lanes 32*(w%4)..: it
    // owns weight rows 32*(w%4)+lane of every matrix of its team's steps.
    const int g = warp & 3, team = (warp - TC_WARP_DQ0) >> 2;
    const int r = 32 * g + lane;
    const uint32_t lane_addr = (uint32_t)(32 * g) << 16;
    uint32_t j = 0, gs0 = 0;  // team K-steps so far; K-steps of earlier tiles
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
      int e, ntok, slot0;
      if (!tc_tile(p, routed_tt, tile / RT, e, ntok, slot0)) continue;
      for (int ks = team; ks < KSTEPS; ks += 2, ++j) {
        const uint32_t gs = gs0 + ks;               // global K-step
        const uint32_t rit = gs >> 2;               // raw slot sequence (4 K-steps a slot)
        const int rs = rit % RS, st = team * 2 + (int)(j & 1u);
        if ((ks & 3) == team)                       // this warp's first step of the slot
          if (!(ok = tc_wait_warp(raw_full + rs, (rit / RS) & 1u, abort_s, lane))) break;
        if (!(ok = tc_wait_warp(a_empty + st, ((j >> 1) & 1u) ^ 1u, abort_s, lane))) break;
        tc::tc_fence_after();
        const uint8_t *raw = sm + L::OFF_RAW + rs * L::RAWSL;
        const uint32_t acol = tmem + lane_addr + (uint32_t)(TM::A_COL0 + st * NA * 32);
#pragma unroll
        for (int m = 0; m < NA; ++m) {
          uint32_t o[32];
          const uint8_t *blk = raw + (m * TC_M + r) * Q4K_BYTES;
          tc_dequant_sub(blk, ks & 3, 0, o);
          tc_dequant_sub(blk, ks & 3, 1, o + 16);
          tc::tmem_st32(acol + (uint32_t)(m * 32), o);
        }
        tc::tmem_wait_st();
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(a_full + st);
        if ((ks & 3) == 2 + team)                   // this warp's last step of the slot
          if (lane == 0) tc::mbar_arrive(raw_empty + rs);
      }
      gs0 += KSTEPS;
    }
  }

  // ---------------- teardown ----------------
  __syncthreads();
  if (*abort_s) {
    if (tid == 0) atomicOr(p.status, DEV_ERR_TIMEOUT);
    for (int i = 0; i < 1000; ++i) __nanosleep(1000);  // let in-flight TMA/MMA land (~1 ms)
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (warp == 0) tc::tmem_dealloc(tmem, TC_TMEM_COLS);
}

// xg[slot][H] = f16(x[token of slot]) for every slot whose expert runs on the
// tensor-core path: routed slot s holds entry order[s] (token order[s] / k,
// expert ids[order[s]]); slot n + t is the shared expert's row of token t.
// One CTA per slot; slots of CUDA-core experts are skipped.
__global__ void __launch_bounds__(256) gather_f16_kernel(const float *__restrict__ x, int H,
                                                         const int32_t *__restrict__ order,
                                                         const int32_t *__restrict__ ids,
                                                         const int32_t *__restrict__ counts,
                                                         int thr, int n, int k, int shared_tc,
                                                         __half *__restrict__ xg) {
  const int slot = blockIdx.x;
  int tok;
  if (slot < n) {
    const int entry = order[slot];
    if (counts[ids[entry]] < thr) return;
    tok = entry / k;
  } else {
    if (!shared_tc) return;
    tok = slot - n;
  }
  const float4 *src = reinterpret_cast<const float4 *>(x + (int64_t)tok * H);
  uint2 *dst = reinterpret_cast<uint2 *>(xg + (int64_t)slot * H);
  for (int i = threadIdx.x; i < H / 4; i += blockDim.x) {
    const float4 v = src[i];
    const __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
    dst[i] = make_uint2(*reinterpret_cast<const uint32_t *>(&a), *reinterpret_cast<const uint32_t *>(&b));
  }
}

int32_t launch_gather_f16(har_cuda_ctx *ctx, const float *x, int H, const int32_t *order,
                          const int32_t *ids, const int32_t *counts, int thr, int n, int k,
                          int T, int shared_tc, __half *xg) {
  prof_begin(ctx);
  gather_f16_kernel<<<n + T, 256, 0, ctx->stream>>>(x, H, order, ids, counts, thr, n, k,
                                                    shared_tc, xg);
  return check_launch(ctx, "gather_f16_kernel");
}

int32_t launch_moe_tc(har_cuda_ctx *ctx, const TcMaps &maps, const TcParams &p, int na,
                      int max_tiles) {
  const int grid = std::max(1, std::min(ctx->num_sms, max_tiles));
  if (na == 2) {
    const size_t smem = (size_t)TcSmem<2>::BYTES + 1024;
    cudaFuncSetAttribute(moe_tc_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    prof_begin(ctx);
    moe_tc_kernel<2><<<grid, TC_THREADS, smem, ctx->stream>>>(maps, p);
    return check_launch(ctx, "moe_tc_gate_up_kernel");
  }
  const size_t smem = (size_t)TcSmem<1>::BYTES + 1024;
  cudaFuncSetAttribute(moe_tc_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  prof_begin(ctx);
  moe_tc_kernel<1><<<grid, TC_THREADS, smem, ctx->stream>>>(maps, p);
  return check_launch(ctx, "moe_tc_down_kernel");
}

}  // namespace har
