// k_moe_tc_f16w.cu — the opt-in fast variant of the tensor-core expert
// path (HAR_CUDA_MOE_TC_F16W): each dequantised Q4_K weight is rounded once
// to f16, w = d*sc*(q - 8) + (8*d*sc - dmin*m), and a tile's K-steps
// accumulate into one TMEM accumulator, so the epilogue runs once per tile.
// Activations are hi/lo f16 pairs as on the default path.  Results meet the
// north star's max relative error 1e-3 (about 4e-4 of max|y| measured), not
// HAR's normalised-RMS verdict of 5e-5, which the default path
// (k_moe_tc.cu) meets; in exchange the dequantisation is a plain per-weight
// formula with no per-super-block accumulator hand-off.
//
// Roles and pipeline are those of k_moe_tc.cu (tc_pipeline.cuh): raw Q4_K
// boxes by TMA into a shared-memory ring, 16 dequant warps in four teams
// writing f16 weight stages into tensor memory, one MMA warp, and here four
// epilogue warps (one per TMEM lane group) handling a whole tile at its end.
// No multicast: every TMA load reads this GPU's memory into this CTA only.
#include <algorithm>

#include "gemv_engine.cuh"
#include "tc_pipeline.cuh"

namespace har {

constexpr int F16W_WARP_DQ0 = 7;  // warps 3..6 epilogue, 7..22 dequantisers
constexpr int F16W_THREADS = 32 * (F16W_WARP_DQ0 + TC_DQ_WARPS);

// Shared-memory plan: raw ring (one super-block step = 4 K-steps per slot)
// and B ring (16 KB slots of 128/box-rows K-steps).  The f16 weight operand
// does not touch shared memory: it is written to tensor memory.
template <int NA>
struct F16wSmem {
  static constexpr int RAW_SLOTS = NA == 2 ? 4 : 6;
  static constexpr int B_SLOTS = 4;
  static constexpr int BSL = 128 * 128;           // 16 KB: 128 rows of 64 f16
  static constexpr int RAWSL = NA * TC_M * Q4K_BYTES;
  static constexpr int OFF_B = 0;                 // 1024-aligned swizzled buffers first
  static constexpr int OFF_RAW = OFF_B + B_SLOTS * BSL;
  static constexpr int BYTES = OFF_RAW + RAW_SLOTS * RAWSL;
};

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
__device__ __forceinline__ void f16w_dequant_step(const uint8_t *blk, int c, uint32_t (&o)[32]) {
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

// Position of K index k: see tc_kperm (tc_pipeline.cuh).

// NA = number of A matrices (2: gate and up with SwiGLU epilogue; 1: one
// matrix, the fallback for a down GEMM whose H is not a multiple of 256).
// PAIR (NA = 2): the down GEMM with its two "matrices" the row blocks
// [r0, r0 + 128) and [r0 + 128, r0 + 256) of one weight tensor; a tile covers
// 256 output rows, and the epilogue writes both accumulators to ybuf.
template <int NA, bool PAIR>
__global__ void __launch_bounds__(F16W_THREADS, 1) moe_tc_f16w_kernel(const __grid_constant__ TcMaps maps,
                                                               const TcParams p) {
  using L = F16wSmem<NA>;
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
  } else if (warp < F16W_WARP_DQ0) {
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
              if (!(fabsf(av) < 65520.0f)) atomicOr(p.status, DEV_ERR_RANGE);  // beyond f16 (or NaN)
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
    const int g = warp & 3, team = (warp - F16W_WARP_DQ0) >> 2;
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
          f16w_dequant_step(raw + (m * TC_M + r) * Q4K_BYTES, team, o);
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

int32_t launch_moe_tc_f16w(har_cuda_ctx *ctx, const TcMaps &maps, const TcParams &p, int na,
                      int max_tiles) {
  const int grid = std::max(1, std::min(ctx->num_sms, max_tiles));
  if (na == 2) {
    const size_t smem = (size_t)F16wSmem<2>::BYTES + 1024;
    cudaFuncSetAttribute(moe_tc_f16w_kernel<2, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    prof_begin(ctx);
    moe_tc_f16w_kernel<2, false><<<grid, F16W_THREADS, smem, ctx->stream>>>(maps, p);
    return check_launch(ctx, "moe_tc_f16w_gate_up_kernel");
  }
  if (p.rows % (2 * TC_M) == 0) {
    // the down GEMM as 256-row tiles: two 128-row blocks share each token tile
    const size_t smem = (size_t)F16wSmem<2>::BYTES + 1024;
    cudaFuncSetAttribute(moe_tc_f16w_kernel<2, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    prof_begin(ctx);
    moe_tc_f16w_kernel<2, true><<<grid, F16W_THREADS, smem, ctx->stream>>>(maps, p);
    return check_launch(ctx, "moe_tc_f16w_down_kernel");
  }
  const size_t smem = (size_t)F16wSmem<1>::BYTES + 1024;
  cudaFuncSetAttribute(moe_tc_f16w_kernel<1, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  prof_begin(ctx);
  moe_tc_f16w_kernel<1, false><<<grid, F16W_THREADS, smem, ctx->stream>>>(maps, p);
  return check_launch(ctx, "moe_tc_f16w_down_kernel");
}

}  // namespace har
