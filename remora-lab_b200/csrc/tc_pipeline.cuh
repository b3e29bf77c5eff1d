// tc_pipeline.cuh — the pieces the tensor-core expert kernels share: the
// tensor-memory plan, the accumulator ring, the bounded mbarrier waits and
// the MMA issuer's K-step loop (one warp, one elected lane issues).
#pragma once

#include "moe_tc.cuh"
#include "tc_ptx.cuh"

namespace har {

// Tensor-memory plan (512 columns x 128 lanes): accumulators in 64-column
// quarters at [0, A_COL0), then one f16 weight stage per dequant team of
// SW = NA x 32 columns (one 64-value K-step of each matrix: row = lane, two
// f16 per column).  A super-block unit of a tile whose token box has bw B
// rows (2 per token) takes ceil(NA * bw / 64) quarters: matrix m's
// accumulator sits at column m * bw of the unit's first quarter.
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

// Accumulator quarters of the next unit: `qc` is the ring cursor (the MMA
// warp and the epilogue walk the same units, so they agree); a unit that does
// not fit before the end wraps to quarter 0.  Returns the first quarter.
template <typename TM>
__device__ __forceinline__ int tc_take_quarters(int &qc, int nq) {
  if (qc + nq > TM::NQ) qc = 0;
  const int q0 = qc;
  qc += nq;
  if (qc == TM::NQ) qc = 0;
  return q0;
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

}  // namespace har
