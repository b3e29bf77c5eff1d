// moe_tc.cuh — parameters shared by the expert-FFN executor (k_moe.cu) and
// its tensor-core path (k_moe_tc.cu).
#pragma once

#include <cuda_fp16.h>

#include "har_internal.cuh"

namespace har {

constexpr int TC_M = 128;   // weight rows per tile (MMA M)
constexpr int TC_NT = 32;   // tokens per tile (two MMA N columns each: hi and lo)
constexpr int TC_NBOX = 2;  // token-tile boxes of 32 and 64 rows (16 and 32 tokens)
constexpr int TC_KS = 128;  // H and I must be multiples of this
constexpr uint32_t TC_WAIT_LIMIT = 1u << 22;  // polls before a wait is declared stuck

// Warp roles of the tensor-core kernel.
constexpr int TC_WARP_TMA = 0;    // one thread: TMA loads of raw weight boxes
constexpr int TC_WARP_MMA = 1;    // the MMA issuer (whole warp, one elected lane issues)
constexpr int TC_WARP_BTMA = 2;   // one thread: TMA loads of token tiles
constexpr int TC_WARP_EPI0 = 3;   // warps 3..10: TMEM -> registers -> global epilogue
constexpr int TC_EPI_WARPS = 8;   // two per TMEM lane group: tokens 0..15 and 16..31 of a tile
constexpr int TC_WARP_DQ0 = TC_WARP_EPI0 + TC_EPI_WARPS;  // warps 11..26: dequantisers
constexpr int TC_DQ_TEAMS = 4;    // four warps each; team t fills weight stage t
constexpr int TC_DQ_WARPS = 4 * TC_DQ_TEAMS;
constexpr int TC_WARPS = TC_WARP_DQ0 + TC_DQ_WARPS;
constexpr int TC_THREADS = 32 * TC_WARPS;
constexpr int TC_TMEM_COLS = 512;  // accumulators, then the f16 weight stages

struct TcParams {
  int rows;        // weight rows per expert (I for gate/up, H for down)
  int K;           // reduction length (H for gate/up, I for down)
  int E, T, k, n;
  int shared_tc;   // the shared expert runs on this path
  const int2 *tt_info;    // token tiles: {expert (E = shared) | tokens << 16, first slot}
  const int32_t *n_tt;    // number of token tiles
  __half *a16;     // gate/up output [2 * slots][I]: f16 hi/lo row pairs
  float *ybuf;     // down output [slots][H]
  int out_ld;      // row length of the output (I or H)
  int *status;
  // The epilogue reads each super-block's d and dmin (its unit's scale) from
  // the weights themselves: matrix 0/1 of the routed experts
  // ([E*rows][row_bytes]) and of the shared expert ([rows][row_bytes]).
  const uint8_t *w0, *w1, *sw0, *sw1;
  int64_t row_bytes;
  __half *s16_out;  // gate/up: the down GEMM's min-term operand, [2 * slots][I/16]
};

// TMA maps of one launch: the A matrices (routed [E*rows][row_bytes] and the
// shared expert's [rows][row_bytes], 128 x 144-byte boxes) and the B operand
// ([2 * slots][K] f16: slot s is rows 2s (hi) and 2s+1 (lo), 64-value boxes
// of 32/64 rows, 128-byte swizzle: a tile loads the smallest box that covers
// its tokens).
// The s16 maps cover the min-term operand of the B rows ([2 * slots][K/16]
// f16: row 2s / 2s + 1 holds the hi / lo part of slot s's 32-value sub-block
// sums, each twice), in boxes of 32/64 rows x 8 values (half a super-block).
struct TcMaps {
  TmaDesc a0, a1, sh0, sh1;
  TmaDesc b[TC_NBOX];    // token-tile boxes of 32 and 64 rows (16 and 32 tokens)
  TmaDesc s16[TC_NBOX];  // the same rows' min-term operand
};

int32_t launch_moe_tc(har_cuda_ctx *ctx, const TcMaps &maps, const TcParams &p, int na,
                      int max_tiles);
// The same GEMMs with each dequantised weight rounded to f16 (k_moe_tc_f16w.cu).
int32_t launch_moe_tc_f16w(har_cuda_ctx *ctx, const TcMaps &maps, const TcParams &p, int na,
                           int max_tiles);
// xg[2 slot], xg[2 slot + 1] = f16 hi/lo of x[token of slot] for the slots of
// experts on the tensor-core path.
// n_valid = the number of grouped entries (offsets[E]); later routed slots are empty.
int32_t launch_gather_f16(har_cuda_ctx *ctx, const float *x, int H, const int32_t *order,
                          const int32_t *ids, const int32_t *counts, const int32_t *n_valid,
                          int thr, int n, int k, int sh0, int shT, int shared_tc, __half *xg, __half *xs16,
                          const float *gi, float *gsh);

}  // namespace har
