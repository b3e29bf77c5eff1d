// moe_tc.cuh — parameters shared by the expert-FFN executor (k_moe.cu) and
// its tensor-core path (k_moe_tc.cu).
#pragma once

#include <cuda_fp16.h>

#include "har_internal.cuh"

namespace har {

constexpr int TC_M = 128;   // weight rows per tile (MMA M)
constexpr int TC_NT = 64;   // token columns per tile (MMA N, max)
constexpr int TC_NBOX = 3;  // token-tile boxes of 16, 32 and 64 rows
constexpr int TC_KS = 128;  // H and I must be multiples of this
constexpr uint32_t TC_WAIT_LIMIT = 1u << 22;  // polls before a wait is declared stuck

// Warp roles of the tensor-core kernel.
constexpr int TC_WARP_TMA = 0;    // one thread: TMA loads of raw weight boxes
constexpr int TC_WARP_MMA0 = 1;   // MMA issuer of the even K-steps
constexpr int TC_WARP_BTMA = 2;   // one thread: TMA loads of token tiles
constexpr int TC_WARP_EPI0 = 3;   // warps 3..6: TMEM -> global epilogue (one per lane group)
constexpr int TC_WARP_DQ0 = 7;    // warps 7..14: dequantise raw Q4_K into f16 weight stages
constexpr int TC_DQ_WARPS = 8;
constexpr int TC_WARP_MMA1 = 15;  // MMA issuer of the odd K-steps
constexpr int TC_ISSUERS = 2;
constexpr int TC_WARPS = 16;
constexpr int TC_THREADS = 32 * TC_WARPS;
constexpr int TC_TMEM_COLS = 512;  // accumulators, then the f16 weight stages

struct TcParams {
  int rows;        // weight rows per expert (I for gate/up, H for down)
  int K;           // reduction length (H for gate/up, I for down)
  int E, T, k, n;
  int shared_tc;   // the shared expert runs on this path
  const int2 *tt_info;    // routed token tiles: {expert | tokens << 16, first slot}
  const int32_t *n_tt;    // number of routed token tiles
  __half *a16;     // gate/up output [slots][I]
  float *ybuf;     // down output [slots][H]
  int out_ld;      // row length of the output (I or H)
  int *status;
};

// TMA maps of one launch: the A matrices (routed [E*rows][row_bytes] and the
// shared expert's [rows][row_bytes], 128 x 144-byte boxes) and the B operand
// ([slots][K] f16 in slot order, 64-value boxes of 16/32/64 rows, 128-byte
// swizzle: a tile loads the smallest box that covers its tokens).
struct TcMaps {
  TmaDesc a0, a1, sh0, sh1;
  TmaDesc b[TC_NBOX];  // token-tile boxes of 16, 32 and 64 rows
};

int32_t launch_moe_tc(har_cuda_ctx *ctx, const TcMaps &maps, const TcParams &p, int na,
                      int max_tiles);
// xg[slot][H] = f16(x[token of slot]) for the slots of experts on the tensor-core path.
int32_t launch_gather_f16(har_cuda_ctx *ctx, const float *x, int H, const int32_t *order,
                          const int32_t *ids, const int32_t *counts, int thr, int n, int k,
                          int T, int shared_tc, __half *xg);

}  // namespace har
