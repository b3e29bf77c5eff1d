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
// ~22 significant bits and only the weights are rounded to f16; the epilogue
// adds the two accumulator columns.  D = W_tile * X^T accumulates in TMEM (f32).
//   gate/up: two accumulators (gate rows and up rows of the same 128
//            intermediate indices); epilogue a = silu(g) * u -> a16 (hi/lo f16
//            rows of the slot, the down GEMM's B operand).
//   down:    one accumulator; epilogue ybuf[slot][h] (f32), then the common
//            combine kernel applies the routing weights in slot order.
//
// With few tokens per expert the MMAs are narrow (N = 32..64) and issue
// rate matters: one SM's share of HBM bandwidth is ~40 Q4_K weights per cycle,
// and a K-step (NA x 4 MMAs of 128 x 16 weights) must issue in ~400 cycles.
// The issuing warp stays warp-uniform, elects its lane once and issues a
// K-step's MMAs from one asm block (~40 cycles per MMA, measured).
//
// One persistent CTA per SM, warp-specialised, every handoff an mbarrier:
//   TMA threads:  one loads raw Q4_K boxes (128 rows x one 144-byte
//                 super-block per matrix) into a raw ring in shared memory;
//                 another loads 128-byte-swizzled f16 token tiles (64 values x
//                 32/64 rows: the smallest box covering the tile's hi/lo rows,
//                 which sit in slot order) into a B ring whose 16 KB slots
//                 hold 128/box-rows K-steps each.
//   dequant warps: four teams of four, team t taking the K-steps ks = t
//                 (mod 4), turn the raw blocks into f16 weights with packed-f16
//                 arithmetic and store them straight into the team's
//                 tensor-memory stage with tcgen05.st (warp w owns TMEM lanes
//                 32*(w%4).. = those rows).  Keeping the weight operand out of
//                 shared memory keeps its write and its tensor-core read off
//                 the shared-memory bandwidth.  The dequantisation is most of
//                 the kernel's instruction stream, hence the 16 warps.
//   MMA warp:     4 x tcgen05.mma (K=16, A from TMEM, B from shared memory)
//                 per matrix per K-step; tcgen05.commit frees the weight stage
//                 and the B slot, and signals the epilogue at the end of a tile.
//   epilogue warps: tcgen05.ld the accumulator (hi and lo columns of each
//                 token), add, apply the epilogue, store, then free the
//                 accumulator columns.
// No multicast: every TMA load reads this GPU's memory into this CTA only.
// Operands are f16 (same tensor rate as bf16, 3 more mantissa bits): each
// weight is rounded once to f16 from d*sc*(q - 8) (exact) plus a centred
// per-sub-block offset rounded to f16; activations are hi/lo f16 pairs;
// accumulation is f32.
// K order: inside every group of four K values both operands hold positions
// (0, 2, 1, 3) -- the order in which nibble pairs come out of a 32-bit word
// with one mask each -- which leaves every dot product unchanged.
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
// quarters at [0, A_COL0), then one f16 weight stage per dequant team of
// SW = NA x 32 columns (one 64-value K-step of each matrix: row = lane, two
// f16 per column).  A tile whose token box has bw B rows (2 per token) takes
// ceil(NA * bw / 64) quarters: matrix m's accumulator sits at column m * bw
// of the tile's first quarter.
template <int NA>
struct TcTmem {
  static constexpr int A_STAGES = TC_DQ_TEAMS;
  static constexpr int SW = NA * 32;
  static constexpr int A_COL0 = TC_TMEM_COLS - A_STAGES * SW;
  static constexpr int NQ = A_COL0 / 64;
  static __device__ __forceinline__ int quarters(int bw) {
    return (NA * bw + 63) / 64;
  }
};

// Smallest token-tile box covering n tokens: 0 = 32 B rows (16 tokens), 1 = 64.
__device__ __forceinline__ int tc_box(int n) { return n <= 16 ? 0 : 1; }

// Accumulator quarters of the next tile: `qc` is the ring cursor (the MMA
// warps and the epilogue walk the same tiles, so they agree); a tile that does
// not fit before the end wraps to quarter 0.  Returns the first quarter.
template <typename TM>
__device__ __forceinline__ int tc_take_quarters(int &qc, int nq) {
  if (qc + nq > TM::NQ) qc = 0;
  const int q0 = qc;
  qc += nq;
  if (qc == TM::NQ) qc = 0;
  return q0;
}

// Dequantise one 64-value K-step (chunk c of 4) of a raw Q4_K block in
// shared memory (`blk` = the 144-byte block of this lane's row) into 32 f16x2
// words: o[0..16) the low-nibble sub-block 2c, o[16..32) the high-nibble
// sub-block 2c+1, each word-pair holding values (4i, 4i+2), (4i+1, 4i+3).
//
// Each weight is computed centred, w = d*sc*(q - 8) + (8*d*sc - dmin*m):
// the offset c = 8*d*sc - dmin*m sits near the middle of the sub-block's
// range, so rounding it to f16 costs little.  (Rounding the raw offset
// -dmin*m instead, as large as the weights, puts one shared error on all 32
// weights of a sub-block and about doubles the error of a dot product.)
// Packed f16 arithmetic, two values per instruction:
//   a mask and a shift put two nibbles in mantissa bits 4..7 under the
//   exponent of 64: (v & 0x00F000F0) | 0x54005400 = (64 + q0, 64 + q2);
//   hfma2(64 + q, sc, -72 sc) = sc*(q - 8) exactly (|.| <= 504, and 72*sc has
//   at most 10 significant bits);
//   hfma2(sc*(q - 8), d, c) = the weight rounded once to f16 (d is the block's
//   f16 scale, exact; c is rounded to f16 from f32).
__device__ __forceinline__ void tc_dequant_step(const uint8_t *blk, int c, uint32_t (&o)[32]) {
  const uint4 hdr = *reinterpret_cast<const uint4 *>(blk);
  const uint4 qa = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * c);
  const uint4 qb = *reinterpret_cast<const uint4 *>(blk + 32 + 32 * c);
  int sc0, m0, sc1, m1;
  q4k_scale_min(hdr.y, hdr.z, hdr.w, 2 * c, sc0, m0);
  q4k_scale_min(hdr.y, hdr.z, hdr.w, 2 * c + 1, sc1, m1);
  const __half2 d2 = __half2half2(__ushort_as_half((unsigned short)(hdr.x & 0xffffu)));
  const float d = f16_bits_to_f32(hdr.x & 0xffffu), dmin = f16_bits_to_f32(hdr.x >> 16);
  const __half2 s_lo = __half2half2(__int2half_rn(sc0));
  const __half2 n_lo = __half2half2(__int2half_rn(-72 * sc0));
  const __half2 c_lo = __half2half2(__float2half_rn(8.0f * d * (float)sc0 - dmin * (float)m0));
  const __half2 s_hi = __half2half2(__int2half_rn(sc1));
  const __half2 n_hi = __half2half2(__int2half_rn(-72 * sc1));
  const __half2 c_hi = __half2half2(__float2half_rn(8.0f * d * (float)sc1 - dmin * (float)m1));
  const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {  // word i: bytes 4i .. 4i+3 of the chunk
    const uint32_t w = q[i];
    const uint32_t pa = ((w << 4) & 0x00F000F0u) | 0x54005400u;  // low nibbles of bytes 0, 2
    const uint32_t pb = ((w >> 4) & 0x00F000F0u) | 0x54005400u;  // low nibbles of bytes 1, 3
    const uint32_t pc = (w & 0x00F000F0u) | 0x54005400u;         // high nibbles of bytes 0, 2
    const uint32_t pd = ((w >> 8) & 0x00F000F0u) | 0x54005400u;  // high nibbles of bytes 1, 3
    const __half2 a = __hfma2(__hfma2(*reinterpret_cast<const __half2 *>(&pa), s_lo, n_lo), d2, c_lo);
    const __half2 b = __hfma2(__hfma2(*reinterpret_cast<const __half2 *>(&pb), s_lo, n_lo), d2, c_lo);
    const __half2 e = __hfma2(__hfma2(*reinterpret_cast<const __half2 *>(&pc), s_hi, n_hi), d2, c_hi);
    const __half2 f = __hfma2(__hfma2(*reinterpret_cast<const __half2 *>(&pd), s_hi, n_hi), d2, c_hi);
    o[2 * i] = *reinterpret_cast<const uint32_t *>(&a);
    o[2 * i + 1] = *reinterpret_cast<const uint32_t *>(&b);
    o[16 + 2 * i] = *reinterpret_cast<const uint32_t *>(&e);
    o[16 + 2 * i + 1] = *reinterpret_cast<const uint32_t *>(&f);
  }
}

// Position of K index k in the (0, 2, 1, 3)-per-group order of the operands.
__host__ __device__ __forceinline__ int tc_kperm(int k) {
  return (k & ~3) | ((k & 1) << 1) | ((k >> 1) & 1);
}

__device__ __forceinline__ float tc_silu(float v) { return v / (1.0f + expf(-v)); }

// Bounded wait shared by the roles: false (and the CTA-wide abort flag set)
// when the barrier phase did not complete within TC_WAIT_LIMIT polls.
// Waiters with sleep_ns > 0 sleep between polls (up to sleep_ns): the
// producers and the epilogue, off the critical path; the MMA issuer and the
// dequantisers spin.
__device__ __forceinline__ bool tc_wait(uint64_t *bar, uint32_t parity, volatile int *abort_s,
                                        uint32_t sleep_ns = 0) {
  if (*abort_s) return false;
  if (sleep_ns ? tc::mbar_wait_lazy(bar, parity, TC_WAIT_LIMIT, sleep_ns)
               : tc::mbar_wait(bar, parity, TC_WAIT_LIMIT))
    return true;
  *abort_s = 1;
  return false;
}
// The same for a whole warp, which leaves converged (the warp-wide tcgen05
// forms need it so): one warp-wide test first, then lane 0 polls and the
// outcome is broadcast.
__device__ __forceinline__ bool tc_wait_warp(uint64_t *bar, uint32_t parity, volatile int *abort_s,
                                             int lane, uint32_t sleep_ns = 0) {
  if (__all_sync(0xffffffffu, tc::mbar_try_wait(bar, parity))) return true;
  bool ok = true;
  if (lane == 0) ok = tc_wait(bar, parity, abort_s, sleep_ns);
  return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
}

// MMA issuer state carried across tiles.
struct TcIssuer {
  uint32_t lead, b_base, a_base, af, ae;  // af / ae: shared addresses of a_full[0] / a_empty[0]
  uint64_t *a_full, *b_full, *b_empty;
  uint32_t ph;     // phase of the current group of four stages
  uint32_t b_it;   // B slot uses so far
  uint32_t a_rdy;  // non-blocking test of the next K-step's stage
  uint32_t b_rdy;  // ... and of the next B slot
};

// K-step J (0..3) of a group: weight stage J; B slots hold KPB = 128 / BW
// K-steps and a new slot opens when J % KPB == 0.  False when a bounded wait
// gave up.
template <int NA, int BW, typename L, int J>
__device__ __forceinline__ bool tc_issue_kstep(TcIssuer &is, uint32_t dcol, uint32_t idesc, bool first,
                                               uint64_t &bslot, int &bs, volatile int *abort_s, int lane) {
  constexpr int KPB = 128 / BW, BS = L::B_SLOTS;
  constexpr uint32_t SUB = BW * 128 / 16;  // one K-step of B, descriptor units
  constexpr int SW = TcTmem<NA>::SW;
  if (J % KPB == 0) {
    bs = (int)(is.b_it % BS);
    if (!__all_sync(0xffffffffu, is.b_rdy != 0) &&
        !tc_wait_warp(is.b_full + bs, (is.b_it / BS) & 1u, abort_s, lane))
      return false;
    bslot = tc::desc_sw128(is.b_base + (uint32_t)(bs * L::BSL));
    is.b_rdy = tc::mbar_test_wait(is.b_full + (is.b_it + 1u) % BS, ((is.b_it + 1u) / BS) & 1u);
  }
  if (!__all_sync(0xffffffffu, is.a_rdy != 0) && !tc_wait_warp(is.a_full + J, is.ph, abort_s, lane))
    return false;
  tc::tc_fence_after();
  is.a_rdy = tc::mbar_test_wait_at<((J + 1) & 3) * 8>(is.af, J == 3 ? is.ph ^ 1u : is.ph);
  tc::mma_kstep_ts_imm<NA, BW>(is.lead, dcol, is.a_base + (uint32_t)(J * SW),
                               bslot + (uint64_t)((J % KPB) * SUB), idesc, first ? 0u : 1u);
  tc::mma_commit_at<J * 8>(is.lead, is.ae);
  if (J % KPB == KPB - 1) {
    tc::mma_commit_w(is.lead, is.b_empty + bs);
    ++is.b_it;
  }
  return true;
}

// The MMAs of one tile: its K-steps in groups of four, one per weight stage.
// False when a bounded wait gave up.
template <int NA, int BW, typename L>
__device__ __forceinline__ bool tc_issue_tile(TcIssuer &is, uint32_t dcol, uint32_t idesc, int ksteps,
                                              volatile int *abort_s, int lane) {
  uint64_t bslot = 0;
  int bs = 0;
  for (int g = 0; g < ksteps; g += 4) {
    if (!tc_issue_kstep<NA, BW, L, 0>(is, dcol, idesc, g == 0, bslot, bs, abort_s, lane) ||
        !tc_issue_kstep<NA, BW, L, 1>(is, dcol, idesc, false, bslot, bs, abort_s, lane) ||
        !tc_issue_kstep<NA, BW, L, 2>(is, dcol, idesc, false, bslot, bs, abort_s, lane) ||
        !tc_issue_kstep<NA, BW, L, 3>(is, dcol, idesc, false, bslot, bs, abort_s, lane))
      return false;
    is.ph ^= 1u;
  }
  return true;
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
      tc::mbar_init(a_full + s, TC_DQ_WARPS / TC_DQ_TEAMS);  // one team fills a stage
      tc::mbar_init(a_empty + s, 1);
    }
    for (int q = 0; q < NQ; ++q) {
      tc::mbar_init(acc_full + q, 1);
      tc::mbar_init(acc_empty + q, 4);
    }
    for (int s = 0; s < BS; ++s) {
      tc::mbar_init(b_full + s, 1);
      tc::mbar_init(b_empty + s, 1);
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
    // ---------------- producer: token tiles (box sized to the tile) ----------------
    if (lane == 0) {
      uint32_t b_it = 0;
      bool ok = true;
      int2 nxt = p.tt_info[min((int)blockIdx.x, max(total - 1, 0)) / RT];
      for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
        const int2 cur = nxt;  // the next tile's entry is loaded one tile ahead
        nxt = p.tt_info[min(tile + (int)gridDim.x, total - 1) / RT];
        const int ntok = cur.x >> 16, slot0 = cur.y;
        const int bx = tc_box(ntok);
        const void *bm = &maps.b[bx];
        const int bw = 32 << bx, kpb = 128 / bw;  // B rows of the tile; K-steps per B slot
        const uint32_t sub_bytes = (uint32_t)bw * 128u;
        for (int s0 = 0; ok && s0 < KSTEPS; s0 += kpb) {
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
    // (every tile has a multiple of 4 K-steps); its fill completes phase
    // gs / 4 of a_full[gs % 4], and B slot use b_it completes phase b_it / BS
    // of b_full[b_it % BS].  The issuer is the critical path: a single warp
    // whose every instruction between two K-steps' MMAs leaves the tensor
    // pipe idle.  So the K-steps of a tile run as groups of four unrolled
    // over the stages (stage, barrier and column offsets are immediates), and
    // the barrier of the next K-step (and of the next B slot) is tested
    // without blocking before the current MMAs are issued; the blocking wait
    // runs only when that test failed.  A stage (slot) cannot complete its
    // next phase before this warp commits the current one, so an early
    // positive test stays valid.
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
    int qc = 0;
    bool ok = true;
    int2 nxt = p.tt_info[min((int)blockIdx.x, max(total - 1, 0)) / RT];
    for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
      const int2 cur = nxt;  // the next tile's entry is loaded one tile ahead
      nxt = p.tt_info[min(tile + (int)gridDim.x, total - 1) / RT];
      const int ntok = cur.x >> 16;
      const int bw = 32 << tc_box(ntok), nq = TM::quarters(bw);
      const int q0 = tc_take_quarters<TM>(qc, nq);
      for (int u = 0; ok && u < nq; ++u)
        ok = tc_wait_warp(acc_empty + q0 + u, ((par >> (q0 + u)) & 1u) ^ 1u, abort_s, lane);
      if (!ok) break;
      tc::tc_fence_after();
      const uint32_t idesc = tc::idesc_f16(TC_M, (2 * ntok + 15) & ~15);
      const uint32_t dcol = tmem + (uint32_t)(q0 * 64);
      ok = bw == 32 ? tc_issue_tile<NA, 32, L>(is, dcol, idesc, KSTEPS, abort_s, lane)
                    : tc_issue_tile<NA, 64, L>(is, dcol, idesc, KSTEPS, abort_s, lane);
      if (!ok) break;
      for (int u = 0; u < nq; ++u) tc::mma_commit_w(lead, acc_full + q0 + u);
      par ^= ((1u << nq) - 1u) << q0;
    }
  } else if (warp < TC_WARP_DQ0) {
    // ---------------- epilogue: TMEM -> global ----------------
    const int g = warp & 3;  // TMEM lane group this warp may access
    const uint32_t lane_addr = (uint32_t)(32 * g) << 16;
    uint32_t par = 0;
    int qc = 0;
    bool ok = true;
    int2 nxt = p.tt_info[min((int)blockIdx.x, max(total - 1, 0)) / RT];
    for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
      const int2 cur = nxt;  // the next tile's entry is loaded one tile ahead
      nxt = p.tt_info[min(tile + (int)gridDim.x, total - 1) / RT];
      const int ntok = cur.x >> 16, slot0 = cur.y;
      const int bw = 32 << tc_box(ntok), nq = TM::quarters(bw);
      const int q0 = tc_take_quarters<TM>(qc, nq);
      for (int u = 0; ok && u < nq; ++u)
        ok = tc_wait_warp(acc_full + q0 + u, (par >> (q0 + u)) & 1u, abort_s, lane, 256);
      if (!ok) break;
      tc::tc_fence_after();
      const int row = (tile % RT) * (PAIR ? 2 * TC_M : TC_M) + 32 * g + lane;
      const uint32_t dcol = tmem + lane_addr + (uint32_t)(q0 * 64);
      const int prow = tc_kperm(row);  // a16 feeds the down GEMM's K axis
      // column 2t holds token t's hi part, 2t+1 its lo part; 16 columns = 8 tokens
      for (int col = 0; col < 2 * ntok; col += 16) {
        const int t0 = col >> 1;
        uint32_t v[16];
        tc::tmem_ld16(dcol + (uint32_t)col, v);                          // matrix 0
        tc::tmem_wait_ld();
        float gv[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) gv[c] = __uint_as_float(v[2 * c]) + __uint_as_float(v[2 * c + 1]);
        if (PAIR) {
          tc::tmem_ld16(dcol + (uint32_t)(bw + col), v);                 // rows + 128
          tc::tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 8; ++c)
            if (t0 + c < ntok) {
              float *dst = p.ybuf + ((int64_t)slot0 + t0 + c) * p.out_ld + row;
              dst[0] = gv[c];
              dst[TC_M] = __uint_as_float(v[2 * c]) + __uint_as_float(v[2 * c + 1]);
            }
        } else if (NA == 2) {
          tc::tmem_ld16(dcol + (uint32_t)(bw + col), v);                 // matrix 1
          tc::tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 8; ++c)
            if (t0 + c < ntok) {
              const float uv = __uint_as_float(v[2 * c]) + __uint_as_float(v[2 * c + 1]);
              const float av = __fmul_rn(tc_silu(gv[c]), uv);
              const __half hi = __float2half_rn(av);
              const __half lo = __float2half_rn(av - __half2float(hi));
              __half *dst = p.a16 + 2 * ((int64_t)slot0 + t0 + c) * p.out_ld + prow;
              dst[0] = hi;
              dst[p.out_ld] = lo;
            }
        } else {
#pragma unroll
          for (int c = 0; c < 8; ++c)
            if (t0 + c < ntok) p.ybuf[((int64_t)slot0 + t0 + c) * p.out_ld + row] = gv[c];
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
    // Team t (four warps) takes the K-steps ks = t (mod 4) -- one of the four
    // K-steps of every raw slot -- and fills weight stage t with them.  Warp
    // w may store only TMEM lanes 32*(w%4)..: it owns weight rows
    // 32*(w%4)+lane of every matrix.
    const int g = warp & 3, team = (warp - TC_WARP_DQ0) >> 2;
    const int r = 32 * g + lane;
    const uint32_t lane_addr = (uint32_t)(32 * g) << 16;
    const uint32_t acol = tmem + lane_addr + (uint32_t)(TM::A_COL0 + team * TM::SW);
    uint32_t u = 0;  // this team's K-steps so far (and raw slots: one K-step each)
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
      for (int ks = team; ks < KSTEPS; ks += TC_DQ_TEAMS, ++u) {
        const int rs = (int)(u % RS);
        if (!(ok = tc_wait_warp(raw_full + rs, (u / RS) & 1u, abort_s, lane))) break;
        if (!(ok = tc_wait_warp(a_empty + team, (u & 1u) ^ 1u, abort_s, lane))) break;
        tc::tc_fence_after();
        const uint8_t *raw = sm + L::OFF_RAW + rs * L::RAWSL;
#pragma unroll
        for (int m = 0; m < NA; ++m) {  // team t holds chunk t of the super-block
          uint32_t o[32];
          tc_dequant_step(raw + (m * TC_M + r) * Q4K_BYTES, team, o);
          tc::tmem_st32(acol + (uint32_t)(m * 32), o);
        }
        tc::tmem_wait_st();
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          tc::mbar_arrive(a_full + team);
          tc::mbar_arrive(raw_empty + rs);
        }
      }
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

// xg[2 slot] = hi = f16(x[token of slot]) and xg[2 slot + 1] = f16(x - hi),
// K order (0, 2, 1, 3) inside each group of four (the weight operand's order),
// for every slot whose expert runs on the tensor-core path: routed slot s holds entry order[s] (token order[s] / k,
// expert ids[order[s]]); slot n + t is the shared expert's row of token t.
// Slots of CUDA-core experts are skipped.  One warp per slot, GATHER_WARPS
// slots per block: the slot's index chain (order -> ids -> counts) of several
// slots is in flight at once.  The warp of shared slot n + t also writes the
// shared expert's gate gsh[t] = sigmoid(gi . x[t]) when gi is given.
constexpr int GATHER_WARPS = 8;

__global__ void __launch_bounds__(GATHER_WARPS * 32) gather_f16_kernel(
    const float *__restrict__ x, int H, const int32_t *__restrict__ order,
    const int32_t *__restrict__ ids, const int32_t *__restrict__ counts,
    const int32_t *__restrict__ n_valid, int thr, int n, int k, int T, int shared_tc,
    __half *__restrict__ xg, const float *__restrict__ gi, float *__restrict__ gsh) {
  const int slot = blockIdx.x * GATHER_WARPS + (int)(threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (slot >= n + T) return;
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
    tok = slot - n;
  }
  const float4 *src = reinterpret_cast<const float4 *>(x + (int64_t)tok * H);
  uint2 *dhi = reinterpret_cast<uint2 *>(xg + 2 * (int64_t)slot * H);
  uint2 *dlo = dhi + H / 4;
#pragma unroll 4
  for (int i = lane; i < H / 4; i += 32) {
    const float4 v = src[i];  // K order (0, 2, 1, 3) inside each group of four
    const __half2 a = __floats2half2_rn(v.x, v.z), b = __floats2half2_rn(v.y, v.w);
    const float2 fa = __half22float2(a), fb = __half22float2(b);
    const __half2 la = __floats2half2_rn(v.x - fa.x, v.z - fa.y), lb = __floats2half2_rn(v.y - fb.x, v.w - fb.y);
    dhi[i] = make_uint2(*reinterpret_cast<const uint32_t *>(&a), *reinterpret_cast<const uint32_t *>(&b));
    dlo[i] = make_uint2(*reinterpret_cast<const uint32_t *>(&la), *reinterpret_cast<const uint32_t *>(&lb));
  }
  if (slot >= n && gi) {
    const float g = shared_gate_warp(gi, x + (int64_t)tok * H, H, lane);
    if (lane == 0) gsh[tok] = g;
  }
}

int32_t launch_gather_f16(har_cuda_ctx *ctx, const float *x, int H, const int32_t *order,
                          const int32_t *ids, const int32_t *counts, const int32_t *n_valid,
                          int thr, int n, int k, int T, int shared_tc, __half *xg,
                          const float *gi, float *gsh) {
  prof_begin(ctx);
  const unsigned grid = (unsigned)((n + T + GATHER_WARPS - 1) / GATHER_WARPS);
  gather_f16_kernel<<<grid, GATHER_WARPS * 32, 0, ctx->stream>>>(x, H, order, ids, counts, n_valid, thr,
                                                                n, k, T, shared_tc, xg, gi, gsh);
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
