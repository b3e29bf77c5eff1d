// k_moe_tc.cu — the tensor-core path of the expert FFN: grouped per-expert
// gate/up GEMM with fused SwiGLU, and the down GEMM, on tcgen05 for experts
// whose token count reaches a threshold (the rest take the CUDA-core GEMV path
// in k_moe.cu).  Semantics are compose_moe_route's
// (har/crates/har-demo/src/bin/har-native-qwen35moe.rs:979-1048) per token.
//
// Shape: the weights are the MMA's M side ("swap AB"): a tile is 128 weight
// rows x up to 32 tokens, so a tile of W is dequantised once for up to 32
// tokens.  Each token is two B rows, the f16 value and the f16 remainder
// (hi = f16(x), lo = f16(x - hi)), so activations reach the tensor cores with
// ~22 significant bits; the epilogue adds the two accumulator columns.
//
// Numerics (f32-grade: HAR's differential verdict, normalised RMS <= 5e-5,
// holds with a wide margin).  A Q4_K weight of sub-block j of super-block b is
// w = d_b*sc_j*q - dmin_b*m_j (q4k.rs:77-89).  Split the row's dot product by
// super-block:
//   sum_k w_k x_k = sum_b s_b * [ sum_{k in b} (sc_j q_k 2^-e_b) x_k
//                                 + sum_j c_bj S_bj(x) ],
//   s_b = d_b 2^e_b,  c_bj = -m_j dmin_b / s_b,
// S_bj(x) = the sum of x over sub-block j of super-block b.  sc*q*2^-e is a
// small integer times a power of two, exact in f16, so the tensor cores see
// exact weights; the min term is one more K=16 MMA per super-block whose A
// operand is c_bj split into f16 hi + lo (8 x 2 values per row, from shared
// memory) and whose B operand is S_bj split the same way (precomputed per
// token row).  Each super-block accumulates into its own TMEM unit, which the
// epilogue scales by s_b in f32.  e_b >= 0 is the smallest shift that keeps
// |c_bj| < 2^15 (e_b = 0 unless dmin > 512 d); d = 0 drops the sc*q term.
// Nothing is rounded to f16 but the hi/lo splits (~22 bits each).
//   gate/up: two accumulators per unit (gate rows and up rows of the same 128
//            intermediate indices); after the last unit a = silu(g) * u ->
//            a16 (hi/lo f16 rows of the slot, the down GEMM's B operand) and
//            a's sub-block sums (the down GEMM's min-term operand).
//   down:    ybuf[slot][h] (f32); the common combine kernel then applies the
//            routing weights in slot order.
//
// One persistent CTA per SM, warp-specialised, every handoff an mbarrier:
//   TMA threads:  one loads raw Q4_K boxes (128 rows x one 144-byte
//                 super-block per matrix) into a raw ring in shared memory;
//                 another loads 128-byte-swizzled f16 token tiles (64 values x
//                 32/64 rows: the smallest box covering the tile's hi/lo rows,
//                 which sit in slot order) into a B ring whose 16 KB slots
//                 hold 128/box-rows K-steps each, and per super-block the same
//                 rows' min-term operand (16 values each) into an S ring.
//   dequant warps: four teams of four, team t taking the K-steps ks = t
//                 (mod 4), turn the raw blocks into the f16 values sc*q*2^-e
//                 and store them straight into the team's tensor-memory stage
//                 with tcgen05.st (warp w owns TMEM lanes 32*(w%4).. = those
//                 rows); each team also writes c_bj hi/lo of its two
//                 sub-blocks of those rows into a shared-memory A' ring.
//   MMA warp:     per super-block unit, 4 K-steps of 4 x tcgen05.mma (K=16, A
//                 from TMEM, B from shared memory) per matrix into a fresh
//                 accumulator, then the min-term MMA (A' and S from shared
//                 memory); tcgen05.commit frees the stages and slots, and
//                 hands the unit to the epilogue.
//   epilogue warps: eight, two per TMEM lane group (tokens 0..15 and 16..31
//                 of a tile): per unit tcgen05.ld the hi and lo columns and
//                 accumulate s_b * (hi + lo) in registers, then free the unit;
//                 after the tile's last unit, the output.
// No multicast: every TMA load reads this GPU's memory into this CTA only.
// K order: inside every group of four K values both operands hold positions
// (0, 2, 1, 3) -- the order in which nibble pairs come out of a 32-bit word
// with one mask each -- which leaves every dot product unchanged.
#include <algorithm>

#include "gemv_engine.cuh"
#include "tc_pipeline.cuh"

namespace har {

// Shared-memory plan: raw ring (one super-block step = 4 K-steps per slot)
// and B ring (16 KB slots of 128/box-rows K-steps).  The f16 weight operand
// does not touch shared memory: it is written to tensor memory.
template <int NA>
struct TcSmem {
  static constexpr int RAW_SLOTS = NA == 2 ? 4 : 6;
  static constexpr int B_SLOTS = 3;
  static constexpr int S_SLOTS = 4;               // min-term B operands in flight (one per unit)
  static constexpr int AP_SLOTS = 2;              // min-term A operands in flight
  static constexpr int BSL = 128 * 128;           // 16 KB: 128 rows of 64 f16
  static constexpr int RAWSL = NA * TC_M * Q4K_BYTES;
  static constexpr int SSL = 64 * 16 * 2;         // up to 64 B rows x 16 f16 (two 8-value boxes)
  static constexpr int APM = TC_M * 16 * 2;       // one matrix's A': 128 rows x 16 f16
  static constexpr int APSL = NA * APM;
  // The 1024-aligned swizzled B ring first; the small no-swizzle rings next
  // (their descriptors' strides stay well inside the buffer); the raw ring last.
  static constexpr int OFF_B = 0;
  static constexpr int OFF_S = OFF_B + B_SLOTS * BSL;
  static constexpr int OFF_AP = OFF_S + S_SLOTS * SSL;
  static constexpr int OFF_RAW = OFF_AP + AP_SLOTS * APSL;
  static constexpr int BYTES = OFF_RAW + RAW_SLOTS * RAWSL;
  static_assert(OFF_RAW % 1024 == 0, "raw slots start on 1024-byte boundaries");
};

// A super-block's unit scale s = d * 2^e and the factor 2^-e its sc values
// take (0 when d = 0: the sc*q term vanishes and the unit carries only the
// min term, with s = dmin / 512).  e = 0 unless dmin >= 512 |d|; then e is
// taken from the exponent fields so that |dmin / s| < 512 and every
// c_j = -m_j * dmin / s (m_j <= 63) stays below 2^15 in f16.  ok = false when
// that needs e > 20, beyond which sc * 2^-e / 16 is no longer exact in f16 (a
// block whose min offset exceeds 2^29 times its scale step; quantisers do not
// produce one).  The dequant warps and the epilogue both call this on the
// same header word, so they agree bit for bit.
struct TcUnitScale {
  float s, a_mul, dmin;
  bool ok;
};
__device__ __forceinline__ TcUnitScale tc_unit_scale(uint32_t dm) {
  TcUnitScale u;
  const float d = f16_bits_to_f32(dm), dmin = f16_bits_to_f32(dm >> 16);
  u.dmin = dmin;
  u.ok = true;
  if (d != 0.0f) {
    // with |dmin| < 2^(ed+1) and |d| >= 2^er: |dmin / d| < 2^(ed - er + 1) = 2^(e + 9)
    int e = 0;
    if (fabsf(dmin) >= 512.0f * fabsf(d)) {
      const int ed = (int)((__float_as_uint(dmin) >> 23) & 255u), er = (int)((__float_as_uint(d) >> 23) & 255u);
      e = ed - er - 8;
    }
    if (e > 20) {
      u.ok = false;
      e = 20;
    }
    u.s = __fmul_rn(d, __uint_as_float((uint32_t)(127 + e) << 23));
    u.a_mul = __uint_as_float((uint32_t)(127 - e) << 23);
  } else {
    u.s = dmin != 0.0f ? __fmul_rn(dmin, 1.0f / 512.0f) : 1.0f;
    u.a_mul = 0.0f;
  }
  return u;
}

// Dequantise one 64-value K-step (chunk c of 4) of a raw Q4_K block in
// shared memory (`blk` = the 144-byte block of this lane's row) into 32 f16x2
// words of sc*q*2^-e: o[0..16) the low-nibble sub-block 2c, o[16..32) the
// high-nibble sub-block 2c+1, each word-pair holding values (4i, 4i+2),
// (4i+1, 4i+3); and the min-term A operand of those two sub-blocks,
// c_j = -m_j * dmin / s for j = 2c, 2c+1 as f16 (hi, lo) pairs, into ap
// (this row's 32 bytes of the unit's A': K = 2j, 2j + 1 in the K-major
// no-swizzle layout, 8 values per 16-byte core-matrix row).
// Packed f16 arithmetic for the weights, two values per instruction, exact:
//   one mask-and-or puts a nibble pair under the exponent of 1024 (ulp 1):
//   (v & 0x000F000F) | 0x64006400 = (1024 + q0, 1024 + q2) for the low
//   nibbles of bytes 0 and 2, and (v & 0x00F000F0) | 0x64006400 =
//   (1024 + 16 q0', ...) for their high nibbles; bytes 1 and 3 take the same
//   masks on v >> 8;
//   hfma2(1024 + q, f, -1024 f) = f*q and hfma2(1024 + 16 q, f/16, -64 f) = f*q
//   with f = sc * 2^-e: f, f/16, 1024 f and 64 f are exact in f16 (sc <= 63,
//   e <= 20) and so is the result, so the fma's one rounding changes nothing.
// c_j is rounded in f32 (dmin / s through a fast reciprocal, a few ulp) and
// split into f16 hi + lo: ~22 bits, like the activations.
__device__ __forceinline__ void tc_dequant_step(const uint8_t *blk, int c, uint32_t (&o)[32],
                                                uint8_t *ap, bool &range_ok) {
  const uint4 hdr = *reinterpret_cast<const uint4 *>(blk);
  const uint4 qa = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * c);
  const uint4 qb = *reinterpret_cast<const uint4 *>(blk + 32 + 32 * c);
  const TcUnitScale us = tc_unit_scale(hdr.x);
  range_ok &= us.ok;
  int sc0, m0, sc1, m1;
  q4k_scale_min(hdr.y, hdr.z, hdr.w, 2 * c, sc0, m0);
  q4k_scale_min(hdr.y, hdr.z, hdr.w, 2 * c + 1, sc1, m1);
  // the min-term operand of sub-blocks 2c, 2c + 1 (packed conversions: two values each)
  const float qm = __fdividef(us.dmin, us.s);
  const float c0 = -__fmul_rn((float)m0, qm), c1 = -__fmul_rn((float)m1, qm);
  const __half2 hh = __floats2half2_rn(c0, c1);
  const float2 hf = __half22float2(hh);
  const __half2 ll = __floats2half2_rn(__fsub_rn(c0, hf.x), __fsub_rn(c1, hf.y));
  const uint32_t hw = *reinterpret_cast<const uint32_t *>(&hh), lw = *reinterpret_cast<const uint32_t *>(&ll);
  *reinterpret_cast<uint2 *>(ap + (c >> 1) * 128 + (c & 1) * 8) =
      make_uint2(__byte_perm(hw, lw, 0x5410), __byte_perm(hw, lw, 0x7632));  // (hi0, lo0), (hi1, lo1)
  // the weights
  const float f0 = __fmul_rn((float)sc0, us.a_mul), f1 = __fmul_rn((float)sc1, us.a_mul);
  const __half2 s_lo = __float2half2_rn(f0);
  const __half2 n_lo = __float2half2_rn(-1024.0f * f0);
  const __half2 s_hi = __float2half2_rn(0.0625f * f1);
  const __half2 n_hi = __float2half2_rn(-64.0f * f1);
  const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {  // word i: bytes 4i .. 4i+3 of the chunk
    const uint32_t w = q[i], t = w >> 8;
    const uint32_t pa = (w & 0x000F000Fu) | 0x64006400u;  // low nibbles of bytes 0, 2
    const uint32_t pb = (t & 0x000F000Fu) | 0x64006400u;  // low nibbles of bytes 1, 3
    const uint32_t pc = (w & 0x00F000F0u) | 0x64006400u;  // high nibbles of bytes 0, 2
    const uint32_t pd = (t & 0x00F000F0u) | 0x64006400u;  // high nibbles of bytes 1, 3
    const __half2 a = __hfma2(*reinterpret_cast<const __half2 *>(&pa), s_lo, n_lo);
    const __half2 b = __hfma2(*reinterpret_cast<const __half2 *>(&pb), s_lo, n_lo);
    const __half2 e = __hfma2(*reinterpret_cast<const __half2 *>(&pc), s_hi, n_hi);
    const __half2 f = __hfma2(*reinterpret_cast<const __half2 *>(&pd), s_hi, n_hi);
    o[2 * i] = *reinterpret_cast<const uint32_t *>(&a);
    o[2 * i + 1] = *reinterpret_cast<const uint32_t *>(&b);
    o[16 + 2 * i] = *reinterpret_cast<const uint32_t *>(&e);
    o[16 + 2 * i + 1] = *reinterpret_cast<const uint32_t *>(&f);
  }
}

// NA = number of A matrices (2: gate and up with SwiGLU epilogue; 1: one
// matrix, the fallback for a down GEMM whose H is not a multiple of 256).
// PAIR (NA = 2): the down GEMM with its two "matrices" the row blocks
// [r0, r0 + 128) and [r0 + 128, r0 + 256) of one weight tensor; a tile covers
// 256 output rows, and the epilogue writes both accumulators to ybuf.
template <int NA, bool PAIR>
__global__ void __launch_bounds__(TC_THREADS, 1) moe_tc_kernel(const __grid_constant__ TcMaps maps,
                                                               const TcParams p) {
  using L = TcSmem<NA>;
  using TM = TcTmem<NA>;
  static_assert(!PAIR || NA == 2, "row-block pairs run on the two-matrix path");
  extern __shared__ uint8_t tc_raw[];
  constexpr int RS = L::RAW_SLOTS, BS = L::B_SLOTS, SS = L::S_SLOTS, PS = L::AP_SLOTS;
  constexpr int AS = TM::A_STAGES, NQ = TM::NQ;
  __shared__ uint64_t bars[2 * RS + 2 * BS + 2 * AS + 2 * NQ + 2 * SS + 2 * PS];
  uint64_t *raw_full = bars, *raw_empty = bars + RS, *b_full = bars + 2 * RS, *b_empty = bars + 2 * RS + BS;
  uint64_t *a_full = bars + 2 * RS + 2 * BS, *a_empty = a_full + AS;
  uint64_t *acc_full = a_empty + AS, *acc_empty = acc_full + NQ;
  uint64_t *s_full = acc_empty + NQ, *s_empty = s_full + SS;
  uint64_t *ap_full = s_empty + SS, *ap_empty = ap_full + PS;
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
      tc::mbar_init(a_full + s, TC_DQ_WARPS / TC_DQ_TEAMS);  // one team fills a stage
      tc::mbar_init(a_empty + s, 1);
    }
    for (int q = 0; q < NQ; ++q) {
      tc::mbar_init(acc_full + q, 1);
      tc::mbar_init(acc_empty + q, TC_EPI_WARPS);
    }
    for (int s = 0; s < BS; ++s) {
      tc::mbar_init(b_full + s, 1);
      tc::mbar_init(b_empty + s, 1);
    }
    for (int s = 0; s < SS; ++s) {
      tc::mbar_init(s_full + s, 1);
      tc::mbar_init(s_empty + s, 1);
    }
    for (int s = 0; s < PS; ++s) {
      tc::mbar_init(ap_full + s, TC_DQ_WARPS);  // every team writes its sub-blocks of A'
      tc::mbar_init(ap_empty + s, 1);
    }
    tc::fence_mbar_init();
    abort_flag = 0;
  }
  if (tid == 0) {
    tc::tma_prefetch_desc(&maps.a0);
    tc::tma_prefetch_desc(&maps.b[0]);
    tc::tma_prefetch_desc(&maps.s16[0]);
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = tmem_base;

  const int RT = p.rows / (PAIR ? 2 * TC_M : TC_M);
  const int KSTEPS = p.K / 64, KSB = p.K / 256;
  // Tiles: token tile (tile / RT) x weight-row tile (tile % RT), walked with a
  // stride of gridDim.x.  Each role loads the table entry of its next tile one
  // tile ahead, unconditionally (clamped index), so the load stays in flight.
  const int total = *p.n_tt * RT;

  if (warp == TC_WARP_TMA) {
    // ---------------- producer: raw weight boxes ----------------
    if (lane == 0) {
      uint32_t raw_it = 0;
      bool ok = true;
      int2 nxt = p.tt_info[min((int)blockIdx.x, max(total - 1, 0)) / RT];
      for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
        const int2 cur = nxt;  // the next tile's entry is loaded one tile ahead
        nxt = p.tt_info[min(tile + (int)gridDim.x, total - 1) / RT];
        const int e = cur.x & 0xffff;
        const int r0 = (tile % RT) * (PAIR ? 2 * TC_M : TC_M);
        const bool sh = e == p.E;
        const void *m0 = sh ? (const void *)&maps.sh0 : (const void *)&maps.a0;
        const void *m1 = PAIR ? m0 : sh ? (const void *)&maps.sh1 : (const void *)&maps.a1;
        const int ya = sh ? r0 : e * p.rows + r0;
        const int ya1 = PAIR ? ya + TC_M : ya;  // matrix 1's rows
        for (int s = 0; ok && s < KSB; ++s) {
          const int rs = raw_it % RS;
          if (!(ok = tc_wait(raw_empty + rs, ((raw_it / RS) & 1u) ^ 1u, abort_s, 256))) break;
          tc::mbar_expect_tx(raw_full + rs, (uint32_t)L::RAWSL);
          uint8_t *dst = sm + L::OFF_RAW + rs * L::RAWSL;
          tc::tma_load_2d(dst, m0, s * Q4K_BYTES, ya, raw_full + rs);
          if (NA == 2) tc::tma_load_2d(dst + TC_M * Q4K_BYTES, m1, s * Q4K_BYTES, ya1, raw_full + rs);
          ++raw_it;
        }
      }
    }
  } else if (warp == TC_WARP_BTMA) {
    // ---- producer: token tiles (box sized to the tile) and their min-term operands ----
    if (lane == 0) {
      uint32_t b_it = 0, s_it = 0;
      bool ok = true;
      int2 nxt = p.tt_info[min((int)blockIdx.x, max(total - 1, 0)) / RT];
      for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
        const int2 cur = nxt;  // the next tile's entry is loaded one tile ahead
        nxt = p.tt_info[min(tile + (int)gridDim.x, total - 1) / RT];
        const int ntok = cur.x >> 16, slot0 = cur.y;
        const int bx = tc_box(ntok);
        const void *bm = &maps.b[bx];
        const void *sm16 = &maps.s16[bx];
        const int bw = 32 << bx, kpb = 128 / bw;  // B rows of the tile; K-steps per B slot
        const uint32_t sub_bytes = (uint32_t)bw * 128u;
        for (int s0 = 0; ok && s0 < KSTEPS; s0 += kpb) {
          if ((s0 & 3) == 0) {  // a super-block starts: its min-term operand, two 8-value boxes
            const int ss = s_it % SS;
            if (!(ok = tc_wait(s_empty + ss, ((s_it / SS) & 1u) ^ 1u, abort_s, 256))) break;
            tc::mbar_expect_tx(s_full + ss, (uint32_t)(2 * bw * 16));
            uint8_t *sdst = sm + L::OFF_S + ss * L::SSL;
            tc::tma_load_2d(sdst, sm16, 4 * s0, 2 * slot0, s_full + ss);
            tc::tma_load_2d(sdst + bw * 16, sm16, 4 * s0 + 8, 2 * slot0, s_full + ss);
            ++s_it;
          }
          const int bs = b_it % BS, nsub = min(kpb, KSTEPS - s0);
          if (!(ok = tc_wait(b_empty + bs, ((b_it / BS) & 1u) ^ 1u, abort_s, 256))) break;
          tc::mbar_expect_tx(b_full + bs, sub_bytes * (uint32_t)nsub);
          for (int j = 0; j < nsub; ++j)
            tc::tma_load_2d(sm + L::OFF_B + bs * L::BSL + j * sub_bytes, bm, (s0 + j) * 64, 2 * slot0,
                            b_full + bs);
          ++b_it;
        }
      }
    }
  } else if (warp == TC_WARP_MMA) {
    // ---------------- MMA issuer (whole warp, one elected lane issues) ----------------
    // Global K-step gs (over this CTA's tiles) sits in weight stage gs % 4
    // (every unit is 4 K-steps); its fill completes phase gs / 4 of
    // a_full[gs % 4], and B slot use b_it completes phase b_it / BS of
    // b_full[b_it % BS].  The issuer is the critical path: a single warp
    // whose every instruction between two K-steps' MMAs leaves the tensor
    // pipe idle.  So a unit's K-steps run unrolled over the stages (stage,
    // barrier and column offsets are immediates), and the barrier of the next
    // K-step (and of the next B slot) is tested without blocking before the
    // current MMAs are issued; the blocking wait runs only when that test
    // failed.  A stage (slot) cannot complete its next phase before this warp
    // commits the current one, so an early positive test stays valid.
    const uint32_t lead = tc::elect_one();
    TcIssuer is;
    is.lead = lead;
    is.b_base = tc::smem_u32(sm + L::OFF_B);
    is.a_base = tmem + (uint32_t)TM::A_COL0;
    is.af = tc::smem_u32(a_full);
    is.ae = tc::smem_u32(a_empty);
    is.b_full = b_full;
    is.b_empty = b_empty;
    is.a_full = a_full;
    is.ph = 0;
    is.b_it = 0;
    is.a_rdy = tc::mbar_test_wait(a_full, 0);
    is.b_rdy = tc::mbar_test_wait(b_full, 0);
    uint32_t par = 0;  // par bit q: parity of quarter q's uses
    uint32_t un = 0;   // units issued so far (A' slot un % PS, S slot un % SS)
    const uint32_t ap_base = tc::smem_u32(sm + L::OFF_AP), s_base = tc::smem_u32(sm + L::OFF_S);
    int qc = 0;
    bool ok = true;
    int2 nxt = p.tt_info[min((int)blockIdx.x, max(total - 1, 0)) / RT];
    for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
      const int2 cur = nxt;  // the next tile's entry is loaded one tile ahead
      nxt = p.tt_info[min(tile + (int)gridDim.x, total - 1) / RT];
      const int ntok = cur.x >> 16;
      const int bw = 32 << tc_box(ntok), nq = TM::quarters(bw);
      const uint32_t idesc = tc::idesc_f16(TC_M, (2 * ntok + 15) & ~15);
      for (int b = 0; ok && b < KSB; ++b, ++un) {  // one accumulator unit per super-block
        const int q0 = tc_take_quarters<TM>(qc, nq);
        for (int u = 0; ok && u < nq; ++u)
          ok = tc_wait_warp(acc_empty + q0 + u, ((par >> (q0 + u)) & 1u) ^ 1u, abort_s, lane);
        if (!ok) break;
        tc::tc_fence_after();
        const uint32_t dcol = tmem + (uint32_t)(q0 * 64);
        ok = bw == 32 ? tc_issue_tile<NA, 32, L>(is, dcol, idesc, 4, abort_s, lane)
                      : tc_issue_tile<NA, 64, L>(is, dcol, idesc, 4, abort_s, lane);
        if (!ok) break;
        // the min term: A' (the rows' c hi/lo) x S (the tokens' sub-block sums hi/lo), K = 16
        const int ps = (int)(un % PS), ss = (int)(un % SS);
        if (!(ok = tc_wait_warp(ap_full + ps, (un / PS) & 1u, abort_s, lane))) break;
        if (!(ok = tc_wait_warp(s_full + ss, (un / SS) & 1u, abort_s, lane))) break;
        tc::tc_fence_after();
        const uint64_t bdesc = tc::desc_noswz(s_base + (uint32_t)(ss * L::SSL), (uint32_t)bw * 16u, 128u);
#pragma unroll
        for (int m = 0; m < NA; ++m)
          tc::mma_f16_ss_w(lead, dcol + (uint32_t)(m * bw),
                           tc::desc_noswz(ap_base + (uint32_t)(ps * L::APSL + m * L::APM), 128u, 256u),
                           bdesc, idesc);
        tc::mma_commit_w(lead, ap_empty + ps);
        tc::mma_commit_w(lead, s_empty + ss);
        for (int u = 0; u < nq; ++u) tc::mma_commit_w(lead, acc_full + q0 + u);
        par ^= ((1u << nq) - 1u) << q0;
      }
    }
  } else if (warp < TC_WARP_DQ0) {
    // ---------------- epilogue: TMEM -> registers -> global ----------------
    // Warp (g, h): TMEM lanes 32g.. (rows 32g + lane of each matrix), tokens
    // 16h .. 16h + 15 of each tile.  Per unit (super-block b) and matrix m:
    //   acc[m][t] += s_b * (hi + lo)
    // with s_b from the block header's d and dmin (read from the weights one
    // unit ahead: an L2 hit, the raw-weight TMA has just brought the block in).
    const int g = warp & 3, h = (warp - TC_WARP_EPI0) >> 2;
    const uint32_t lane_addr = (uint32_t)(32 * g) << 16;
    uint32_t par = 0;
    int qc = 0;
    bool ok = true;
    int2 nxt = p.tt_info[min((int)blockIdx.x, max(total - 1, 0)) / RT];
    for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
      const int2 cur = nxt;  // the next tile's entry is loaded one tile ahead
      nxt = p.tt_info[min(tile + (int)gridDim.x, total - 1) / RT];
      const int ntok = cur.x >> 16, slot0 = cur.y, e = cur.x & 0xffff;
      const int bw = 32 << tc_box(ntok), nq = TM::quarters(bw);
      const int nmine = min(max(ntok - 16 * h, 0), 16);  // this warp's tokens (warp-uniform)
      const int r0 = (tile % RT) * (PAIR ? 2 * TC_M : TC_M);
      const int row = r0 + 32 * g + lane;
      const bool sh = e == p.E;
      const int64_t grow = sh ? row : (int64_t)e * p.rows + row;
      const uint8_t *hp0 = (sh ? p.sw0 : p.w0) + grow * p.row_bytes;
      const uint8_t *hp1 = PAIR ? hp0 + (int64_t)TC_M * p.row_bytes : (sh ? p.sw1 : p.w1) + grow * p.row_bytes;
      float acc[NA][16];
#pragma unroll
      for (int m = 0; m < NA; ++m)
#pragma unroll
        for (int t = 0; t < 16; ++t) acc[m][t] = 0.0f;
      uint32_t dm0 = __ldg(reinterpret_cast<const uint32_t *>(hp0));
      uint32_t dm1 = NA == 2 ? __ldg(reinterpret_cast<const uint32_t *>(hp1)) : 0u;
      for (int b = 0; ok && b < KSB; ++b) {
        const int q0 = tc_take_quarters<TM>(qc, nq);
        const uint32_t cd0 = dm0, cd1 = dm1;
        if (b + 1 < KSB) {  // the next unit's header words, in flight during this unit
          dm0 = __ldg(reinterpret_cast<const uint32_t *>(hp0 + (int64_t)(b + 1) * Q4K_BYTES));
          if (NA == 2) dm1 = __ldg(reinterpret_cast<const uint32_t *>(hp1 + (int64_t)(b + 1) * Q4K_BYTES));
        }
        for (int u = 0; ok && u < nq; ++u)
          ok = tc_wait_warp(acc_full + q0 + u, (par >> (q0 + u)) & 1u, abort_s, lane, 32);
        if (!ok) break;
        tc::tc_fence_after();
        const uint32_t dcol = tmem + lane_addr + (uint32_t)(q0 * 64) + (uint32_t)(32 * h);
        const float sb0 = tc_unit_scale(cd0).s, sb1 = NA == 2 ? tc_unit_scale(cd1).s : 0.0f;
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          if (4 * c4 >= nmine) break;  // warp-uniform
          // tokens 4c4 .. 4c4+3 (hi, lo) of every matrix: one TMEM round trip per group
          uint32_t v[NA][8];
#pragma unroll
          for (int m = 0; m < NA; ++m) tc::tmem_ld8(dcol + (uint32_t)(m * bw + 8 * c4), v[m]);
          tc::tmem_wait_ld();
#pragma unroll
          for (int m = 0; m < NA; ++m)
#pragma unroll
            for (int c = 0; c < 4; ++c)
              acc[m][4 * c4 + c] = fmaf(m == 0 ? sb0 : sb1,
                                        __uint_as_float(v[m][2 * c]) + __uint_as_float(v[m][2 * c + 1]),
                                        acc[m][4 * c4 + c]);
        }
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0)
          for (int u = 0; u < nq; ++u) tc::mbar_arrive(acc_empty + q0 + u);
        par ^= ((1u << nq) - 1u) << q0;
      }
      if (!ok) break;
      // the tile's outputs: tokens 16h + t < ntok of this warp
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        if (t >= nmine) break;  // warp-uniform
        const int64_t slot = (int64_t)slot0 + 16 * h + t;
        if (PAIR) {
          float *dst = p.ybuf + slot * p.out_ld + row;
          dst[0] = acc[0][t];
          dst[TC_M] = acc[NA - 1][t];
        } else if (NA == 2) {
          const float av = __fmul_rn(tc_silu(acc[0][t]), acc[NA - 1][t]);
          if (!(fabsf(av) < 65520.0f)) atomicOr(p.status, DEV_ERR_RANGE);  // beyond f16 (or NaN)
          const __half hi = __float2half_rn(av);
          const __half lo = __float2half_rn(av - __half2float(hi));
          __half *dst = p.a16 + 2 * slot * p.out_ld + tc_kperm(row);  // a16 feeds the down GEMM's K axis
          dst[0] = hi;
          dst[p.out_ld] = lo;
          // the down GEMM's min-term operand: the sum of a over these 32 rows
          // (one sub-block), hi and lo, each twice
          const float sa = warp_sum(av);
          if (lane == 0) {
            if (!(fabsf(sa) < 65520.0f)) atomicOr(p.status, DEV_ERR_RANGE);
            const __half shi = __float2half_rn(sa);
            const __half slo = __float2half_rn(__fsub_rn(sa, __half2float(shi)));
            const int ld16 = p.out_ld / 16, sbk = (r0 + 32 * g) / 32;
            *reinterpret_cast<uint32_t *>(p.s16_out + 2 * slot * ld16 + 2 * sbk) =
                (uint32_t)__half_as_ushort(shi) * 0x10001u;
            *reinterpret_cast<uint32_t *>(p.s16_out + (2 * slot + 1) * ld16 + 2 * sbk) =
                (uint32_t)__half_as_ushort(slo) * 0x10001u;
          }
        } else {
          p.ybuf[slot * p.out_ld + row] = acc[0][t];
        }
      }
    }
  } else {
    // ---------------- dequantisers: raw Q4_K -> f16 weight stages in TMEM ----------------
    // Team t (four warps) takes the K-steps ks = t (mod 4) -- chunk t of every
    // super-block, so one K-step per unit -- and fills weight stage t with it,
    // and the unit's min-term operand A' for sub-blocks 2t, 2t + 1.  Warp w
    // may store only TMEM lanes 32*(w%4)..: it owns weight rows 32*(w%4)+lane
    // of every matrix.
    const int g = warp & 3, team = (warp - TC_WARP_DQ0) >> 2;
    const int r = 32 * g + lane;
    const uint32_t lane_addr = (uint32_t)(32 * g) << 16;
    const uint32_t acol = tmem + lane_addr + (uint32_t)(TM::A_COL0 + team * TM::SW);
    uint8_t *ap_row = sm + L::OFF_AP + (r >> 3) * 256 + (r & 7) * 16;
    uint32_t u = 0;  // this team's K-steps so far = units so far (and raw slots: one each)
    bool ok = true, range_ok = true;
    for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
      for (int ks = team; ks < KSTEPS; ks += TC_DQ_TEAMS, ++u) {
        const int rs = (int)(u % RS), ps = (int)(u % PS);
        if (!(ok = tc_wait_warp(raw_full + rs, (u / RS) & 1u, abort_s, lane))) break;
        if (!(ok = tc_wait_warp(ap_empty + ps, ((u / PS) & 1u) ^ 1u, abort_s, lane))) break;
        if (!(ok = tc_wait_warp(a_empty + team, (u & 1u) ^ 1u, abort_s, lane))) break;
        tc::tc_fence_after();
        const uint8_t *raw = sm + L::OFF_RAW + rs * L::RAWSL;
#pragma unroll
        for (int m = 0; m < NA; ++m) {  // team t holds chunk t of the super-block
          uint32_t o[32];
          tc_dequant_step(raw + (m * TC_M + r) * Q4K_BYTES, team, o, ap_row + ps * L::APSL + m * L::APM,
                          range_ok);
          tc::tmem_st32(acol + (uint32_t)(m * 32), o);
        }
        tc::tmem_wait_st();
        tc::fence_proxy_async_smem();  // the A' stores (generic proxy), seen by the tensor core
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          tc::mbar_arrive(a_full + team);
          tc::mbar_arrive(ap_full + ps);
          tc::mbar_arrive(raw_empty + rs);
        }
      }
    }
    if (!__all_sync(0xffffffffu, range_ok) && lane == 0) atomicOr(p.status, DEV_ERR_RANGE);
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

// xg[2 slot] = hi = f16(x[token of slot]) and xg[2 slot + 1] = f16(x - hi),
// K order (0, 2, 1, 3) inside each group of four (the weight operand's order),
// for every slot whose expert runs on the tensor-core path: routed slot s holds entry order[s] (token order[s] / k,
// expert ids[order[s]]); slot n + j is the shared expert's row of token sh0 + j (j < shT).
// Rows 2 slot and 2 slot + 1 of xs16 [2 slots][H/16] get the f16 hi and lo of
// the slot's 32-value sub-block sums, each twice: the min-term operand.
// Slots of CUDA-core experts are skipped.  One warp per slot, GATHER_WARPS
// slots per block: the slot's index chain (order -> ids -> counts) of several
// slots is in flight at once.  The warp of a shared slot also writes the
// shared expert's gate gsh[t] = sigmoid(gi . x[t]) when gi is given.
constexpr int GATHER_WARPS = 8;

__global__ void __launch_bounds__(GATHER_WARPS * 32) gather_f16_kernel(
    const float *__restrict__ x, int H, const int32_t *__restrict__ order,
    const int32_t *__restrict__ ids, const int32_t *__restrict__ counts,
    const int32_t *__restrict__ n_valid, int thr, int n, int k, int sh0, int shT, int shared_tc,
    __half *__restrict__ xg, __half *__restrict__ xs16, const float *__restrict__ gi,
    float *__restrict__ gsh, int *status) {
  const int slot = blockIdx.x * GATHER_WARPS + (int)(threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (slot >= n + shT) return;
  int tok;
  if (slot < n) {
    // grouped positions past the valid entries (those with an out-of-range
    // expert id are dropped by the grouping) hold no entry
    if (slot >= *n_valid) return;
    const int entry = order[slot];
    if (counts[ids[entry]] < thr) return;
    tok = entry / k;
  } else {
    if (!shared_tc) return;
    tok = sh0 + (slot - n);
  }
  const float4 *src = reinterpret_cast<const float4 *>(x + (int64_t)tok * H);
  uint2 *dhi = reinterpret_cast<uint2 *>(xg + 2 * (int64_t)slot * H);
  uint2 *dlo = dhi + H / 4;
  const int ld16 = H / 16;
  uint32_t *shi = reinterpret_cast<uint32_t *>(xs16 + 2 * (int64_t)slot * ld16);
  uint32_t *slo = reinterpret_cast<uint32_t *>(xs16 + (2 * (int64_t)slot + 1) * ld16);
  float vmax = 0.0f;  // the largest magnitude converted to f16 (overflow check)
#pragma unroll 4
  for (int i = lane; i < H / 4; i += 32) {
    const float4 v = src[i];  // K order (0, 2, 1, 3) inside each group of four
    const __half2 a = __floats2half2_rn(v.x, v.z), b = __floats2half2_rn(v.y, v.w);
    const float2 fa = __half22float2(a), fb = __half22float2(b);
    const __half2 la = __floats2half2_rn(v.x - fa.x, v.z - fa.y), lb = __floats2half2_rn(v.y - fb.x, v.w - fb.y);
    dhi[i] = make_uint2(*reinterpret_cast<const uint32_t *>(&a), *reinterpret_cast<const uint32_t *>(&b));
    dlo[i] = make_uint2(*reinterpret_cast<const uint32_t *>(&la), *reinterpret_cast<const uint32_t *>(&lb));
    // sub-block sums: lanes 8j .. 8j+7 hold the 32 values of sub-block i / 8
    float sum = (v.x + v.y) + (v.z + v.w);
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    sum += __shfl_xor_sync(0xffffffffu, sum, 4);
    vmax = fmaxf(vmax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fmaxf(fabsf(v.z), fabsf(v.w)), fabsf(sum))));
    if ((lane & 7) == 0) {
      const __half hh = __float2half_rn(sum);
      const __half ll = __float2half_rn(__fsub_rn(sum, __half2float(hh)));
      shi[i >> 3] = (uint32_t)__half_as_ushort(hh) * 0x10001u;
      slo[i >> 3] = (uint32_t)__half_as_ushort(ll) * 0x10001u;
    }
  }
  if (__any_sync(0xffffffffu, !(vmax < 65520.0f)) && lane == 0) atomicOr(status, DEV_ERR_RANGE);
  if (slot >= n && gi) {
    const float g = shared_gate_warp(gi, x + (int64_t)tok * H, H, lane);
    if (lane == 0) gsh[tok] = g;
  }
}

int32_t launch_gather_f16(har_cuda_ctx *ctx, const float *x, int H, const int32_t *order,
                          const int32_t *ids, const int32_t *counts, const int32_t *n_valid,
                          int thr, int n, int k, int sh0, int shT, int shared_tc, __half *xg,
                          __half *xs16, const float *gi, float *gsh) {
  int *status = ctx->d_status;
  prof_begin(ctx);
  const unsigned grid = (unsigned)((n + shT + GATHER_WARPS - 1) / GATHER_WARPS);
  gather_f16_kernel<<<grid, GATHER_WARPS * 32, 0, ctx->stream>>>(x, H, order, ids, counts, n_valid, thr,
                                                                n, k, sh0, shT, shared_tc, xg, xs16, gi, gsh,
                                                                status);
  return check_launch(ctx, "gather_f16_kernel");
}

int32_t launch_moe_tc(har_cuda_ctx *ctx, const TcMaps &maps, const TcParams &p, int na,
                      int max_tiles) {
  const int grid = std::max(1, std::min(ctx->num_sms, max_tiles));
  if (na == 2) {
    const size_t smem = (size_t)TcSmem<2>::BYTES + 1024;
    cudaFuncSetAttribute(moe_tc_kernel<2, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    prof_begin(ctx);
    moe_tc_kernel<2, false><<<grid, TC_THREADS, smem, ctx->stream>>>(maps, p);
    return check_launch(ctx, "moe_tc_gate_up_kernel");
  }
  if (p.rows % (2 * TC_M) == 0) {
    // the down GEMM as 256-row tiles: two 128-row blocks share each token tile
    const size_t smem = (size_t)TcSmem<2>::BYTES + 1024;
    cudaFuncSetAttribute(moe_tc_kernel<2, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    prof_begin(ctx);
    moe_tc_kernel<2, true><<<grid, TC_THREADS, smem, ctx->stream>>>(maps, p);
    return check_launch(ctx, "moe_tc_down_kernel");
  }
  const size_t smem = (size_t)TcSmem<1>::BYTES + 1024;
  cudaFuncSetAttribute(moe_tc_kernel<1, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  prof_begin(ctx);
  moe_tc_kernel<1, false><<<grid, TC_THREADS, smem, ctx->stream>>>(maps, p);
  return check_launch(ctx, "moe_tc_down_kernel");
}

}  // namespace har
