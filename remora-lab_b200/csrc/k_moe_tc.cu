// k_moe_tc.cu — the tensor-core path of the expert FFN: grouped per-expert
// gate/up GEMM with fused SwiGLU, and the down GEMM, on tcgen05 for experts
// whose token count reaches a threshold (the rest take the CUDA-core GEMV path
// in k_moe.cu).  Semantics are compose_moe_route's
// (har/crates/har-demo/src/bin/har-native-qwen35moe.rs:979-1048) per token.
//
// Shape: the weights are the MMA's M side ("swap AB"): a tile is 128 weight
// rows x up to 128 token columns, so a tile of W is dequantised once for up to
// 128 tokens.  D = W_tile * X^T accumulates in TMEM (f32).
//   gate/up: two accumulators (gate rows and up rows of the same 128
//            intermediate indices); epilogue a = silu(g) * u -> a16[slot][i] (f16).
//   down:    one accumulator; epilogue ybuf[slot][h] (f32), then the common
//            combine kernel applies the routing weights in slot order.
//
// One persistent CTA per SM, warp-specialised, every handoff an mbarrier:
//   TMA threads:  one loads raw Q4_K boxes (128 rows x one 144-byte
//                 super-block per matrix) into a raw ring in shared memory;
//                 another loads 128-byte-swizzled f16 token tiles (64 values x
//                 16/32/64/128 rows: the smallest box covering the tile's
//                 tokens, which sit in slot order) into a B ring whose 16 KB
//                 slots hold 128/box-rows K-steps each.
//   dequant warps: two teams of four take alternate 64-value K-steps, turn
//                 the raw blocks into f16 weights with packed-f16 arithmetic
//                 and store them straight into a tensor-memory stage with
//                 tcgen05.st (warp w owns TMEM lanes 32*(w%4).. = those rows).  Keeping the weight operand
//                 out of shared memory removes its write and its tensor-core
//                 read from the shared-memory bandwidth, which otherwise bounds
//                 this path near 60% of HBM speed.
//   MMA thread:   4 x tcgen05.mma (K=16, A from TMEM, B from shared memory)
//                 per matrix per step into the TMEM accumulator;
//                 tcgen05.commit frees the weight stage and the B slot, and
//                 signals the epilogue at the end of a tile.
//   epilogue warps: tcgen05.ld the accumulator, then free it for the next tile.
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
  static constexpr int BSL = TC_NT * 128;         // 16 KB (a 128-row box)
  static constexpr int RAWSL = NA * TC_M * Q4K_BYTES;
  static constexpr int OFF_B = 0;                 // 1024-aligned swizzled buffers first
  static constexpr int OFF_RAW = OFF_B + B_SLOTS * BSL;
  static constexpr int BYTES = OFF_RAW + RAW_SLOTS * RAWSL;
};

// Tensor-memory plan (512 columns x 128 lanes): the accumulator at columns
// [0, 256) (gate at 0, up at 128; down at 0), then TC_A_STAGES f16 weight
// stages of NA x 32 columns (one 64-value K-step: row = lane, two f16 per
// column in K order).
constexpr int TC_A_STAGES = 4;
constexpr int TC_A_COL0 = 256;

// Smallest token-tile box (16, 32, 64 or 128 rows) covering n tokens.
__device__ __forceinline__ int tc_box(int n) { return n <= 16 ? 0 : n <= 32 ? 1 : n <= 64 ? 2 : 3; }

// Map a tile's token-tile index to (expert or E for shared, first token,
// token count, first slot).  False when the index is past the work.
__device__ __forceinline__ bool tc_tile(const TcParams &p, int tt_global, int &e, int &t0,
                                        int &ntok, int &base) {
  const int nb = *p.n_big;
  const int routed_tt = p.big_tt[nb];
  if (tt_global < routed_tt) {
    int lo = 0, hi = nb - 1;  // last b with big_tt[b] <= tt_global
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (p.big_tt[mid] <= tt_global) lo = mid; else hi = mid - 1;
    }
    e = p.big[lo];
    const int tt = tt_global - p.big_tt[lo];
    t0 = tt * TC_NT;
    ntok = min(TC_NT, p.counts[e] - t0);
    base = p.offsets[e];
    return true;
  }
  if (!p.shared_tc) return false;
  const int tt = tt_global - routed_tt;
  e = p.E;
  t0 = tt * TC_NT;
  ntok = min(TC_NT, p.T - t0);
  base = p.n;
  return ntok > 0;
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

// NA = number of A matrices (2: gate and up with SwiGLU epilogue; 1: down).
template <int NA>
__global__ void __launch_bounds__(TC_THREADS, 1) moe_tc_kernel(const __grid_constant__ TcMaps maps,
                                                               const TcParams p) {
  using L = TcSmem<NA>;
  extern __shared__ uint8_t tc_raw[];
  constexpr int RS = L::RAW_SLOTS, BS = L::B_SLOTS, AS = TC_A_STAGES;
  __shared__ uint64_t bars[2 * RS + 2 * BS + 2 * AS + 4];
  uint64_t *raw_full = bars, *raw_empty = bars + RS, *b_full = bars + 2 * RS, *b_empty = bars + 2 * RS + BS;
  uint64_t *a_full = bars + 2 * RS + 2 * BS, *a_empty = a_full + AS, *acc_full = a_full + 2 * AS;
  uint64_t *acc_empty = acc_full + 2;
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
      tc::mbar_init(a_full + s, TC_DQ_WARPS / 2);  // one team fills a stage
      tc::mbar_init(a_empty + s, 1);
    }
    for (int s = 0; s < 2; ++s) {
      tc::mbar_init(acc_full + s, 1);
      tc::mbar_init(acc_empty + s, 4);
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

  const int RT = p.rows / TC_M;
  const int KSTEPS = p.K / 64, KSB = p.K / 256;
  const int nb = *p.n_big;
  const int total_tt = p.big_tt[nb] + (p.shared_tc ? (p.T + TC_NT - 1) / TC_NT : 0);
  const int total = total_tt * RT;

  if (warp == TC_WARP_TMA) {
    // ---------------- producer: raw weight boxes ----------------
    if (lane == 0) {
      uint32_t raw_it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
        int e, t0, ntok, base;
        if (!tc_tile(p, tile / RT, e, t0, ntok, base)) continue;
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
        int e, t0, ntok, base;
        if (!tc_tile(p, tile / RT, e, t0, ntok, base)) continue;
        const int bx = tc_box(ntok);
        const void *bm = &maps.b[bx];
        const int rows_b = 16 << bx, kpb = 128 / rows_b;  // K-steps per B slot
        const uint32_t sub_bytes = (uint32_t)rows_b * 128u;
        const int yb = base + t0;
        for (int ks = 0; ok && ks < KSTEPS; ks += kpb) {
          const int bs = b_it % BS;
          if (!(ok = tc_wait(b_empty + bs, ((b_it / BS) & 1u) ^ 1u, abort_s))) break;
          tc::mbar_expect_tx(b_full + bs, sub_bytes * (uint32_t)kpb);
          for (int j = 0; j < kpb; ++j)
            tc::tma_load_2d(sm + L::OFF_B + bs * L::BSL + j * sub_bytes, bm, (ks + j) * 64, yb, b_full + bs);
          ++b_it;
        }
      }
    }
  } else if (warp == TC_WARP_MMA) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t a_it = 0, b_it = 0, acc_it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
        int e, t0, ntok, base;
        if (!tc_tile(p, tile / RT, e, t0, ntok, base)) continue;
        const uint32_t idesc = tc::idesc_f16(TC_M, (ntok + 15) & ~15);
        const int rows_b = 16 << tc_box(ntok), kpb = 128 / rows_b;
        const int acc = 0;  // one accumulator buffer; the epilogue frees it
        if (!(ok = tc_wait(acc_empty + acc, (acc_it & 1u) ^ 1u, abort_s))) break;
        tc::tc_fence_after();
        const uint32_t dcol = tmem;
        for (int ks = 0; ok && ks < KSTEPS; ++ks) {
          const int as = a_it % AS, bs = b_it % BS, sub = ks % kpb;
          if (!(ok = tc_wait(a_full + as, (a_it / AS) & 1u, abort_s))) break;
          if (sub == 0)
            if (!(ok = tc_wait(b_full + bs, (b_it / BS) & 1u, abort_s))) break;
          tc::tc_fence_after();
          const uint32_t bbase = tc::smem_u32(sm + L::OFF_B + bs * L::BSL) + (uint32_t)(sub * rows_b * 128);
          const uint32_t acol = tmem + (uint32_t)(TC_A_COL0 + as * NA * 32);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t bdesc = tc::desc_sw128(bbase + 32u * kk);
#pragma unroll
            for (int m = 0; m < NA; ++m)
              tc::mma_f16_ts(dcol + (uint32_t)(m * TC_NT), acol + (uint32_t)(m * 32 + kk * 8), bdesc,
                             idesc, (ks > 0 || kk > 0) ? 1u : 0u);
          }
          tc::mma_commit(a_empty + as);
          ++a_it;
          if (sub == kpb - 1) {
            tc::mma_commit(b_empty + bs);
            ++b_it;
          }
        }
        if (!ok) break;
        tc::mma_commit(acc_full + acc);
        ++acc_it;
      }
    }
  } else if (warp < TC_WARP_DQ0) {
    // ---------------- epilogue: TMEM -> global ----------------
    const int g = warp & 3;  // TMEM lane group this warp may access
    const uint32_t lane_addr = (uint32_t)(32 * g) << 16;
    uint32_t acc_it = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
      int e, t0, ntok, base;
      if (!tc_tile(p, tile / RT, e, t0, ntok, base)) continue;
      const int acc = 0;
      if (!tc_wait(acc_full + acc, acc_it & 1u, abort_s)) break;
      tc::tc_fence_after();
      const int row = (tile % RT) * TC_M + 32 * g + lane;
      const int64_t slot0 = base + t0;
      const uint32_t dcol = tmem + lane_addr;
      for (int col = 0; col < ntok; col += 16) {
        uint32_t v0[16];
        tc::tmem_ld16(dcol + (uint32_t)col, v0);
        if (NA == 2) {
          uint32_t v1[16];
          tc::tmem_ld16(dcol + (uint32_t)(TC_NT + col), v1);
          tc::tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (col + j < ntok) {
              const float av = __fmul_rn(tc_silu(__uint_as_float(v0[j])), __uint_as_float(v1[j]));
              p.a16[(slot0 + col + j) * p.out_ld + row] = __float2half_rn(av);
            }
        } else {
          tc::tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (col + j < ntok) p.ybuf[(slot0 + col + j) * p.out_ld + row] = __uint_as_float(v0[j]);
        }
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(acc_empty + acc);
      ++acc_it;
    }
  } else {
    // ---------------- dequantisers: raw Q4_K -> f16 weight stages in TMEM ----------------
    // Two teams of four warps take alternate K-steps, so two weight stages
    // are filled at once.  Warp w may store only TMEM lanes 32*(w%4)..: it
    // owns weight rows 32*(w%4)+lane of every matrix of its team's steps.
    const int g = warp & 3, team = (warp - TC_WARP_DQ0) >> 2;
    const int r = 32 * g + lane;
    const uint32_t lane_addr = (uint32_t)(32 * g) << 16;
    uint32_t gs0 = 0;  // K-steps of earlier tiles (every tile has a multiple of 4)
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
      int e, t0, ntok, base;
      if (!tc_tile(p, tile / RT, e, t0, ntok, base)) continue;
      for (int ks = team; ok && ks < KSTEPS; ks += 2) {
        const uint32_t gs = gs0 + ks;               // global K-step = A stage sequence
        const uint32_t rit = gs >> 2;               // raw slot sequence
        const int rs = rit % RS, as = gs % AS;
        if ((ks & 3) == team)                       // this warp's first step of the slot
          if (!(ok = tc_wait(raw_full + rs, (rit / RS) & 1u, abort_s))) break;
        if (!(ok = tc_wait(a_empty + as, ((gs / AS) & 1u) ^ 1u, abort_s))) break;
        tc::tc_fence_after();
        const uint8_t *raw = sm + L::OFF_RAW + rs * L::RAWSL;
        const uint32_t acol = tmem + lane_addr + (uint32_t)(TC_A_COL0 + as * NA * 32);
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
        if (lane == 0) tc::mbar_arrive(a_full + as);
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
