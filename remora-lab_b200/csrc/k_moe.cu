// k_moe.cu — the expert-FFN executor: compose_moe_route for a batch of
// tokens, expert-major (har/crates/har-demo/src/bin/har-native-qwen35moe.rs:979-1048
// for the arithmetic, har/crates/har-serve/src/moe.rs:182-255 for the
// grouping that reads each routed expert's weights once per step).
//
// Pipeline on one stream (all device-side; the host never reads counts):
//   1. group_kernel: stable counting sort of the T*k (token, slot) entries by
//      expert; list of non-empty experts.
//   2. [Q8_K mode] quantise the T token rows once.
//   3. moe_gate_up_kernel: for each (expert, tile of intermediate rows), the
//      gate and up GEMV rows for all of the expert's tokens, SwiGLU in
//      registers: a[slot][i] = silu(gate_i . x) * (up_i . x).
//   4. [Q8_K mode] quantise the a rows.
//   5. moe_down_kernel: ybuf[slot][h] = down_h . a[slot] per (expert, tile of
//      hidden rows).
//   6. moe_combine_kernel: per token, routed = sum over slots in slot order of
//      w * down (the reference's `*output += weight * value`), then
//      + sigmoid(gate_inp . x) * shared, then + x with ADD_RESIDUAL.  The
//      combine uses separately rounded multiplies and adds like Rust.
// Slot numbering: routed entries occupy grouped positions [0, n), n = T*k;
// the shared expert's row for token t is slot n + t.
#include <stdlib.h>

#include <algorithm>
#include <climits>

#include "gemv_engine.cuh"
#include "moe_tc.cuh"

namespace har {

size_t group_smem_bytes(int E);
int32_t launch_group_full(har_cuda_ctx *ctx, const int32_t *ids, int64_t n, int E,
                          int32_t *counts, int32_t *offsets, int32_t *order, int32_t *inv,
                          int32_t *ne, int32_t *n_ne, int thr, int nt, int2 *tt_info,
                          int32_t *n_tt, int shared_T, int allow_empty, int32_t *gcnt);

struct MoeDev {
  const uint8_t *gate, *up, *down, *sh_gate, *sh_up, *sh_down;
  int64_t ebytes_gu, ebytes_d;  // bytes per expert
  int64_t rb_h, rb_i;           // Q4_K row bytes for K = H and K = I
  int64_t xrow, arow;           // activation row bytes (f32 or Q8_K) for H and I
  int E, H, I, T, k, n;
  int has_shared;   // the layer has a shared expert (combine adds it)
  int sh0, shT;     // it serves tokens sh0 .. sh0 + shT - 1 (slots n .. n + shT - 1)
  int gemv_shared;  // the shared expert runs on the CUDA-core path
  const int32_t *counts, *offsets, *order, *inv, *ne, *n_ne;
  const uint8_t *xact;  // x rows (f32) or their Q8_K image
  float *a;             // [n + T][I] f32
  const uint8_t *aact;  // a rows (f32, = a) or their Q8_K image
  float *ybuf;          // [n + T][H] f32
  const float *gsh;     // [T] sigmoid(gate_inp . x[t]) of the shared expert, or null (gate 1)
};

// gsh[t] = sigmoid(gi . x[t]), one warp per token: the shared expert's gate,
// computed before any kernel of the layer writes y (which may alias x).
__global__ void __launch_bounds__(256) shared_gate_kernel(const float *__restrict__ gi,
                                                          const float *__restrict__ x, int H, int t0,
                                                          int count, float *__restrict__ gsh) {
  const int j = blockIdx.x * 8 + (int)(threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (j >= count) return;
  const int t = t0 + j;
  const float g = shared_gate_warp(gi, x + (int64_t)t * H, H, lane);
  if (lane == 0) gsh[t] = g;
}

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + expf(-v)); }


// Resolve group gi's expert id, token count and first slot.
__device__ __forceinline__ void group_info(const MoeDev &p, int gi, int nne, int &g, int &cnt,
                                           int &base) {
  if (gi < nne) {
    g = p.ne[gi];
    cnt = p.counts[g];
    base = p.offsets[g];
  } else {
    g = p.E;  // shared expert
    cnt = p.shT;
    base = p.n;
  }
}

// Fill the CTA's token table for tokens [tt, tt+MT) of a group.
template <int MT>
__device__ __forceinline__ void token_table(const MoeDev &p, int g, int cnt, int base, int tt,
                                            const uint8_t *act, int64_t arow, bool by_slot,
                                            const uint8_t **rowp, int *slot) {
  if (threadIdx.x < MT) {
    const int idx = tt + threadIdx.x;
    if (idx < cnt) {
      int s, tok;
      if (g == p.E) {
        tok = p.sh0 + idx;
        s = p.n + idx;
      } else {
        tok = p.order[base + idx] / p.k;
        s = base + idx;
      }
      rowp[threadIdx.x] = act + (int64_t)(by_slot ? s : tok) * arow;
      slot[threadIdx.x] = s;
    } else {
      rowp[threadIdx.x] = nullptr;
      slot[threadIdx.x] = -1;
    }
  }
  __syncthreads();
}

template <int ACT, int LPR, int CPL, int MT>
__global__ void __launch_bounds__(256) moe_gate_up_kernel(MoeDev p, int rows_per_tile) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ const uint8_t *rowp[MT];
  __shared__ int slot[MT];
  constexpr int RPW = 32 / LPR;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = lane / LPR, gl = lane % LPR;
  const int C = p.H / 64;
  const int ntg = (p.I + rows_per_tile - 1) / rows_per_tile;
  const int nne = *p.n_ne;
  const int total = (nne + p.gemv_shared) * ntg;
  for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
    const int gi = tile / ntg, j = tile - gi * ntg;
    int g, cnt, base;
    group_info(p, gi, nne, g, cnt, base);
    const uint8_t *wg = g == p.E ? p.sh_gate : p.gate + (int64_t)g * p.ebytes_gu;
    const uint8_t *wu = g == p.E ? p.sh_up : p.up + (int64_t)g * p.ebytes_gu;
    const int r0 = j * rows_per_tile, r1 = min(p.I, r0 + rows_per_tile);
    for (int tt = 0; tt < cnt; tt += MT) {
      token_table<MT>(p, g, cnt, base, tt, p.xact, p.xrow, false, rowp, slot);
      if (ACT == ACT_F32)
        stage_f32(smem, reinterpret_cast<const float *const *>(rowp), MT, p.H);
      else
        stage_q8k(smem, rowp, MT, p.H);
      LaneAct<ACT> a[MT][CPL];
#pragma unroll
      for (int t = 0; t < MT; ++t)
#pragma unroll
        for (int i = 0; i < CPL; ++i) {
          const int ch = gl + LPR * i;
          if (ch < C) a[t][i].load(smem, MT, p.H, t, ch);
        }
      for (int rb = r0 + warp * RPW; rb < r1; rb += 8 * RPW) {
        const int r = rb + grp;
        const bool valid = r < r1;
        const int rr = valid ? r : rb;
        const uint8_t *rg = wg + (int64_t)rr * p.rb_h;
        const uint8_t *ru = wu + (int64_t)rr * p.rb_h;
        float ag[MT], au[MT];
#pragma unroll
        for (int t = 0; t < MT; ++t) ag[t] = au[t] = 0.0f;
#pragma unroll
        for (int i = 0; i < CPL; ++i) {
          const int ch = gl + LPR * i;
          if (ch < C) {
            const WChunk w1 = load_wchunk(rg, ch);
            const WChunk w2 = load_wchunk(ru, ch);
#pragma unroll
            for (int t = 0; t < MT; ++t) {
              ag[t] += chunk_dot(w1, ch, a[t][i]);
              au[t] += chunk_dot(w2, ch, a[t][i]);
            }
          }
        }
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          ag[t] = lane_group_sum<LPR>(ag[t]);
          au[t] = lane_group_sum<LPR>(au[t]);
        }
        if (valid && gl == 0) {
#pragma unroll
          for (int t = 0; t < MT; ++t)
            if (slot[t] >= 0) p.a[(int64_t)slot[t] * p.I + r] = __fmul_rn(silu_f(ag[t]), au[t]);
        }
      }
      __syncthreads();  // smem and the token table are rewritten next pass
    }
  }
}

template <int ACT, int LPR, int CPL, int MT>
__global__ void __launch_bounds__(256) moe_down_kernel(MoeDev p, int rows_per_tile) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ const uint8_t *rowp[MT];
  __shared__ int slot[MT];
  constexpr int RPW = 32 / LPR;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = lane / LPR, gl = lane % LPR;
  const int C = p.I / 64;
  const int ntg = (p.H + rows_per_tile - 1) / rows_per_tile;
  const int nne = *p.n_ne;
  const int total = (nne + p.gemv_shared) * ntg;
  for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
    const int gi = tile / ntg, j = tile - gi * ntg;
    int g, cnt, base;
    group_info(p, gi, nne, g, cnt, base);
    const uint8_t *wd = g == p.E ? p.sh_down : p.down + (int64_t)g * p.ebytes_d;
    const int r0 = j * rows_per_tile, r1 = min(p.H, r0 + rows_per_tile);
    for (int tt = 0; tt < cnt; tt += MT) {
      token_table<MT>(p, g, cnt, base, tt, p.aact, p.arow, true, rowp, slot);
      if (ACT == ACT_F32)
        stage_f32(smem, reinterpret_cast<const float *const *>(rowp), MT, p.I);
      else
        stage_q8k(smem, rowp, MT, p.I);
      LaneAct<ACT> a[MT][CPL];
#pragma unroll
      for (int t = 0; t < MT; ++t)
#pragma unroll
        for (int i = 0; i < CPL; ++i) {
          const int ch = gl + LPR * i;
          if (ch < C) a[t][i].load(smem, MT, p.I, t, ch);
        }
      for (int rb = r0 + warp * RPW; rb < r1; rb += 8 * RPW) {
        const int r = rb + grp;
        const bool valid = r < r1;
        const uint8_t *rd = wd + (int64_t)(valid ? r : rb) * p.rb_i;
        float acc[MT];
#pragma unroll
        for (int t = 0; t < MT; ++t) acc[t] = 0.0f;
#pragma unroll
        for (int i = 0; i < CPL; ++i) {
          const int ch = gl + LPR * i;
          if (ch < C) {
            const WChunk w = load_wchunk(rd, ch);
#pragma unroll
            for (int t = 0; t < MT; ++t) acc[t] += chunk_dot(w, ch, a[t][i]);
          }
        }
#pragma unroll
        for (int t = 0; t < MT; ++t) acc[t] = lane_group_sum<LPR>(acc[t]);
        if (valid && gl == 0) {
#pragma unroll
          for (int t = 0; t < MT; ++t)
            if (slot[t] >= 0) p.ybuf[(int64_t)slot[t] * p.H + r] = acc[t];
        }
      }
      __syncthreads();
    }
  }
}

// One block per (token, chunk of COMB_T float4 columns): more blocks than
// tokens keep enough loads in flight, and each thread loads the rows of up
// to eight slots before it adds them -- in slot order, as the reference does.
constexpr int COMB_T = 128;

__global__ void __launch_bounds__(COMB_T) moe_combine_kernel(MoeDev p, const float *x,
                                                             const float *__restrict__ weights,
                                                             float *y, int add_residual) {
  // x may alias y (in-place layer stacks): each thread reads x[t] only at the
  // four columns it writes, and the shared expert's gate was computed from x
  // by an earlier kernel (p.gsh), so no block reads what a sibling wrote.
  constexpr int SLOTS = 32;  // slots of the token cached in shared memory
  __shared__ int spos[SLOTS];
  __shared__ float sw[SLOTS];
  const int64_t t = blockIdx.x;
  const float *xt = x + t * p.H;
  const float g = p.gsh ? p.gsh[t] : 1.0f;
  for (int s = threadIdx.x; s < p.k && s < SLOTS; s += blockDim.x) {
    spos[s] = p.inv[t * p.k + s];
    sw[s] = weights[t * p.k + s];
  }
  __syncthreads();
  // four consecutive h per thread (float4); per element the same operation
  // order as the reference: slots in order, then the shared expert, then x
  const int H4 = p.H / 4;
  const int h = blockIdx.y * COMB_T + threadIdx.x;
  if (h >= H4) return;
  const float4 *yb4 = reinterpret_cast<const float4 *>(p.ybuf);
  float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  for (int s0 = 0; s0 < p.k; s0 += 8) {
    float4 v[8];
    float wv[8];
    unsigned used = 0;  // bit j: slot s0 + j holds a row
#pragma unroll
    for (int j = 0; j < 8; ++j) {  // the loads first: up to eight in flight
      const int s = s0 + j;
      int pos = -1;
      wv[j] = 0.0f;
      if (s < p.k) {
        pos = s < SLOTS ? spos[s] : p.inv[t * p.k + s];
        wv[j] = s < SLOTS ? sw[s] : weights[t * p.k + s];
      }
      v[j] = pos >= 0 ? yb4[(int64_t)pos * H4 + h] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      used |= (pos >= 0 ? 1u : 0u) << j;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (!((used >> j) & 1u)) continue;
      acc.x = __fadd_rn(acc.x, __fmul_rn(wv[j], v[j].x));
      acc.y = __fadd_rn(acc.y, __fmul_rn(wv[j], v[j].y));
      acc.z = __fadd_rn(acc.z, __fmul_rn(wv[j], v[j].z));
      acc.w = __fadd_rn(acc.w, __fmul_rn(wv[j], v[j].w));
    }
  }
  if (p.has_shared && t >= p.sh0 && t < p.sh0 + p.shT) {
    const float4 v = yb4[(int64_t)(p.n + t - p.sh0) * H4 + h];
    acc.x = __fadd_rn(acc.x, __fmul_rn(g, v.x));
    acc.y = __fadd_rn(acc.y, __fmul_rn(g, v.y));
    acc.z = __fadd_rn(acc.z, __fmul_rn(g, v.z));
    acc.w = __fadd_rn(acc.w, __fmul_rn(g, v.w));
  }
  if (add_residual) {
    const float4 xv = reinterpret_cast<const float4 *>(xt)[h];
    acc.x = __fadd_rn(xv.x, acc.x);
    acc.y = __fadd_rn(xv.y, acc.y);
    acc.z = __fadd_rn(xv.z, acc.z);
    acc.w = __fadd_rn(xv.w, acc.w);
  }
  reinterpret_cast<float4 *>(y + t * p.H)[h] = acc;
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

template <typename K>
static void set_smem(K kern, size_t smem) {
  if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
}

// Rows per work tile: 4 warp passes for gate/up, 2 for down.
static int rows_per_tile_gu(int H) { return 8 * gemv_shape(H).RPW * 4; }
static int rows_per_tile_d(int I) { return 8 * gemv_shape(I).RPW * 2; }

template <int ACT, int LPR, int CPL, int MT>
static int32_t launch_gate_up(har_cuda_ctx *ctx, const MoeDev &p, int grid) {
  const int rows_per_tile = rows_per_tile_gu(p.H);
  auto kern = moe_gate_up_kernel<ACT, LPR, CPL, MT>;
  const size_t smem = ActSmem<ACT>::bytes(MT, p.H);
  set_smem(kern, smem);
  prof_begin(ctx);
  kern<<<grid, 256, smem, ctx->stream>>>(p, rows_per_tile);
  return check_launch(ctx, "moe_gate_up_kernel");
}

template <int ACT, int LPR, int CPL, int MT>
static int32_t launch_down(har_cuda_ctx *ctx, const MoeDev &p, int grid) {
  const int rows_per_tile = rows_per_tile_d(p.I);
  auto kern = moe_down_kernel<ACT, LPR, CPL, MT>;
  const size_t smem = ActSmem<ACT>::bytes(MT, p.I);
  set_smem(kern, smem);
  prof_begin(ctx);
  kern<<<grid, 256, smem, ctx->stream>>>(p, rows_per_tile);
  return check_launch(ctx, "moe_down_kernel");
}

template <int ACT>
static int32_t dispatch_gate_up(har_cuda_ctx *ctx, const MoeDev &p, int grid) {
  const GemvShape s = gemv_shape(p.H);
  constexpr int M1 = ACT == ACT_Q8K ? 4 : 1;
  constexpr int M2 = ACT == ACT_Q8K ? 2 : 1;
  if (s.LPR == 4) return launch_gate_up<ACT, 4, 1, M1>(ctx, p, grid);
  if (s.LPR == 8) return launch_gate_up<ACT, 8, 1, M1>(ctx, p, grid);
  if (s.LPR == 16) return launch_gate_up<ACT, 16, 1, M1>(ctx, p, grid);
  if (s.CPL == 1) return launch_gate_up<ACT, 32, 1, M1>(ctx, p, grid);
  if (s.CPL == 2) return launch_gate_up<ACT, 32, 2, M2>(ctx, p, grid);
  return set_error(ctx, HAR_CUDA_ERR_UNSUPPORTED, "moe_ffn: hidden size above 4096");
}

template <int ACT>
static int32_t dispatch_down(har_cuda_ctx *ctx, const MoeDev &p, int grid) {
  const GemvShape s = gemv_shape(p.I);
  constexpr int M1 = ACT == ACT_Q8K ? 4 : 1;
  constexpr int M2 = ACT == ACT_Q8K ? 2 : 1;
  if (s.LPR == 4) return launch_down<ACT, 4, 1, M1>(ctx, p, grid);
  if (s.LPR == 8) return launch_down<ACT, 8, 1, M1>(ctx, p, grid);
  if (s.LPR == 16) return launch_down<ACT, 16, 1, M1>(ctx, p, grid);
  if (s.CPL == 1) return launch_down<ACT, 32, 1, M1>(ctx, p, grid);
  if (s.CPL == 2) return launch_down<ACT, 32, 2, M2>(ctx, p, grid);
  return set_error(ctx, HAR_CUDA_ERR_UNSUPPORTED, "moe_ffn: intermediate size above 4096");
}

static size_t al256(size_t v) { return (v + 255) & ~(size_t)255; }

// Scratch layout of one moe_ffn call (offsets in bytes, 256-byte aligned).
struct MoeScratch {
  size_t o_counts, o_offsets, o_order, o_inv, o_ne, o_nne, o_xq, o_a, o_aq, o_y;
  size_t o_ttinfo, o_ntt, o_x16, o_a16, o_xs16, o_as16, o_gsh, o_gcnt, total;
};

// Experts with at least this many tokens take the tensor-core path
// (FORCE_TC: every expert, FORCE_GEMV: none).  The default, 1, sends every
// expert there: measured on the config-5 stack (Zipf top-10 over 512 experts,
// most experts with 1..16 tokens), the tensor-core kernels beat the CUDA-core
// GEMV kernels even for single-token experts.  har_cuda_ctx_set_tc_min_tokens
// overrides it per context, HAR_CUDA_TC_MIN_TOKENS in the environment per process.
// A single-token call would be ~5% faster on the CUDA-core GEMVs (routed
// 48-layer stack: 3.24 against 3.42 ms per step), but the default keeps every
// call on one path so that a token's result does not depend on the batch it
// came in, bit for bit (batched equals isolated, har-serve/src/moe.rs:301-314).
static int tc_threshold(const har_cuda_ctx *ctx, uint32_t flags, int64_t T) {
  (void)T;
  if (flags & HAR_CUDA_MOE_FORCE_TC) return 1;
  if (flags & HAR_CUDA_MOE_FORCE_GEMV) return INT_MAX;
  if (ctx->tc_min_tokens > 0) return ctx->tc_min_tokens;
  static const int thr = [] {
    const char *v = getenv("HAR_CUDA_TC_MIN_TOKENS");
    const int t = v ? atoi(v) : 0;
    return t > 0 ? t : 0;
  }();
  return thr > 0 ? thr : 1;
}

// Whether the layer's shapes fit the tensor-core kernels (H and I multiples
// of 128, TMA maps encoded at layer creation).
static bool tc_shapes_ok(const har_cuda_moe_layer *layer) {
  return layer->tc_maps && layer->H % TC_M == 0 && layer->I % TC_M == 0 &&
         layer->H % TC_KS == 0 && layer->I % TC_KS == 0;
}

// Whether any expert of a call can take the tensor-core path: f32 activation
// semantics (Q8_K calls stay on the GEMV kernels, whose integer dots are the
// Q8_K semantics), the shapes fit, and the threshold is reachable (a token
// routes to an expert at most once, the shared expert sees all T tokens).
// Layers whose shapes do not fit run every expert on the GEMV kernels unless
// FORCE_TC asks for tensor cores.
static bool tc_possible(const har_cuda_ctx *ctx, const har_cuda_moe_layer *layer, int64_t T, int k,
                        uint32_t flags) {
  if (flags & HAR_CUDA_MOE_ACT_Q8K) return false;
  if (!tc_shapes_ok(layer) && !(flags & HAR_CUDA_MOE_FORCE_TC)) return false;
  return (int64_t)tc_threshold(ctx, flags, T) <= T;  // an expert sees each token at most once
}

static MoeScratch moe_layout(const har_cuda_moe_layer *layer, int64_t T, int k, bool q8,
                             bool tc) {
  const int64_t E = layer->E, H = layer->H, I = layer->I;
  const int64_t n = T * k, slots = n + T;
  const int64_t xq_row = (H / QK) * Q8K_BYTES, aq_row = (I / QK) * Q8K_BYTES;
  MoeScratch s;
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off += al256(bytes); return o; };
  s.o_counts = take(4 * (size_t)E);
  s.o_offsets = take(4 * (size_t)(E + 1));
  s.o_order = take(4 * (size_t)n);
  s.o_inv = take(4 * (size_t)n);
  s.o_ne = take(4 * (size_t)E);
  s.o_nne = take(4);
  s.o_xq = q8 ? take((size_t)(T * xq_row)) : 0;
  s.o_a = take(4 * (size_t)(slots * I));
  s.o_aq = q8 ? take((size_t)(slots * aq_row)) : 0;
  s.o_y = take(4 * (size_t)(slots * H));
  // token tiles: routed (<= one partial tile per expert) then the shared expert's
  s.o_ttinfo = take(8 * (size_t)(std::min<int64_t>(E, n) + n / TC_NT + T / TC_NT + 2));
  s.o_ntt = take(4);
  s.o_x16 = tc ? take(4 * (size_t)(slots * H)) : 0;  // token rows in slot order (f16 hi/lo)
  s.o_a16 = tc ? take(4 * (size_t)(slots * I)) : 0;
  // min-term operands of the B rows: [2 * slots][K/16] f16
  s.o_xs16 = tc ? take(2 * (size_t)(2 * slots * (H / 16))) : 0;
  s.o_as16 = tc ? take(2 * (size_t)(2 * slots * (I / 16))) : 0;
  s.o_gsh = take(4 * (size_t)T);
  const size_t gw = group_scratch_words(n, (int)E);  // the multi-CTA grouping's segment counts
  s.o_gcnt = gw ? take(4 * gw) : 0;
  s.total = off;
  return s;
}

size_t moe_scratch_bytes(const har_cuda_ctx *ctx, const har_cuda_moe_layer *layer, int64_t T, int k,
                         uint32_t flags) {
  if (flags & HAR_CUDA_MOE_DECODE) return moe_decode_scratch_bytes(layer, T, k);
  return moe_layout(layer, T, k, (flags & HAR_CUDA_MOE_ACT_Q8K) != 0,
                    tc_possible(ctx, layer, T, k, flags))
      .total;
}

int32_t run_moe_ffn(har_cuda_ctx *ctx, const har_cuda_moe_layer *layer, const float *x,
                    int64_t T, int k, const int32_t *ids, const float *weights, float *y,
                    uint32_t flags) {
  int32_t st = ensure_scratch(ctx, moe_scratch_bytes(ctx, layer, T, k, flags));
  if (st) return st;
  return run_moe_ffn_in(ctx, layer, x, T, k, ids, weights, y, flags, (uint8_t *)ctx->scratch);
}

// The pipeline on a caller-provided scratch region of moe_scratch_bytes()
// bytes; allocates nothing.  Every scratch word is written before it is read.
int32_t run_moe_ffn_in(har_cuda_ctx *ctx, const har_cuda_moe_layer *layer, const float *x,
                       int64_t T, int k, const int32_t *ids, const float *weights, float *y,
                       uint32_t flags, uint8_t *S) {
  return run_moe_ffn_range(ctx, layer, x, T, k, ids, weights, y, flags, S, 0, T);
}

// The same with the shared expert serving only tokens sh0 .. sh0 + shT - 1 of
// the call (the expert-parallel local layer: the shared expert runs on the
// rank's own rows among the received ones); the other tokens get the routed
// sum alone.
int32_t run_moe_ffn_range(har_cuda_ctx *ctx, const har_cuda_moe_layer *layer, const float *x,
                          int64_t T, int k, const int32_t *ids, const float *weights, float *y,
                          uint32_t flags, uint8_t *S, int64_t sh0, int64_t shT) {
  if (flags & HAR_CUDA_MOE_DECODE) {
    if (sh0 != 0 || shT != T)
      return set_error(ctx, HAR_CUDA_ERR_UNSUPPORTED, "moe_ffn: the decode path serves the shared expert on every token");
    return run_moe_decode(ctx, layer, x, T, k, ids, weights, y, flags, S);
  }
  if (sh0 < 0 || shT < 0 || sh0 + shT > T)
    return set_error(ctx, HAR_CUDA_ERR_ARG, "moe_ffn: shared-expert token range outside the call");
  if (((uintptr_t)x & 15u) || ((uintptr_t)y & 15u))
    return set_error(ctx, HAR_CUDA_ERR_ARG, "moe_ffn: x and y must be 16-byte aligned");
  const bool q8 = (flags & HAR_CUDA_MOE_ACT_Q8K) != 0;
  const int E = (int)layer->E, H = (int)layer->H, I = (int)layer->I;
  const int64_t n = T * k;
  const int has_sh = layer->sh_gate ? 1 : 0;
  const int64_t xq_row = (int64_t)(H / QK) * Q8K_BYTES, aq_row = (int64_t)(I / QK) * Q8K_BYTES;
  const bool tc = tc_possible(ctx, layer, T, k, flags);
  const bool f16w = (flags & HAR_CUDA_MOE_TC_F16W) != 0;  // the f16-weight tensor-core variant
  const int thr = tc ? tc_threshold(ctx, flags, T) : INT_MAX;
  const bool shared_tc = has_sh && tc && shT >= thr;
  if (tc && ((H % TC_M) || (I % TC_M) || (H % TC_KS) || (I % TC_KS)))
    return set_error(ctx, HAR_CUDA_ERR_UNSUPPORTED,
                     "moe_ffn: the tensor-core path needs H and I multiples of 128");
  const MoeScratch L = moe_layout(layer, T, k, q8, tc);
  const size_t o_counts = L.o_counts, o_offsets = L.o_offsets, o_order = L.o_order;
  const size_t o_inv = L.o_inv, o_ne = L.o_ne, o_nne = L.o_nne, o_xq = L.o_xq, o_a = L.o_a;
  const size_t o_aq = L.o_aq, o_y = L.o_y;
  int32_t st;
  MoeDev p;
  p.gate = layer->gate->dev;
  p.up = layer->up->dev;
  p.down = layer->down->dev;
  p.sh_gate = has_sh ? layer->sh_gate->dev : nullptr;
  p.sh_up = has_sh ? layer->sh_up->dev : nullptr;
  p.sh_down = has_sh ? layer->sh_down->dev : nullptr;
  p.ebytes_gu = layer->gate->expert_bytes;
  p.ebytes_d = layer->down->expert_bytes;
  p.rb_h = layer->gate->row_bytes;
  p.rb_i = layer->down->row_bytes;
  p.E = E;
  p.H = H;
  p.I = I;
  p.T = (int)T;
  p.k = k;
  p.n = (int)n;
  p.has_shared = has_sh && shT > 0;
  p.sh0 = (int)sh0;
  p.shT = (int)shT;
  p.gemv_shared = has_sh && shT > 0 && !shared_tc;
  p.counts = (const int32_t *)(S + o_counts);
  p.offsets = (const int32_t *)(S + o_offsets);
  p.order = (const int32_t *)(S + o_order);
  p.inv = (const int32_t *)(S + o_inv);
  p.ne = (const int32_t *)(S + o_ne);
  p.n_ne = (const int32_t *)(S + o_nne);
  p.a = (float *)(S + o_a);
  p.ybuf = (float *)(S + o_y);
  // the shared expert's gate: by the gather kernel when it visits the shared
  // slots (tensor-core shared expert), else by its own kernel, before y is written
  const bool gate_row = has_sh && layer->sh_gate_inp;
  p.gsh = gate_row ? (const float *)(S + L.o_gsh) : nullptr;
  if (q8) {
    p.xact = S + o_xq;
    p.xrow = xq_row;
    p.aact = S + o_aq;
    p.arow = aq_row;
  } else {
    p.xact = (const uint8_t *)x;
    p.xrow = (int64_t)H * 4;
    p.aact = (const uint8_t *)p.a;
    p.arow = (int64_t)I * 4;
  }
  st = launch_group_full(ctx, ids, n, E, (int32_t *)(S + o_counts), (int32_t *)(S + o_offsets),
                         (int32_t *)(S + o_order), (int32_t *)(S + o_inv), (int32_t *)(S + o_ne),
                         (int32_t *)(S + o_nne), thr, TC_NT, (int2 *)(S + L.o_ttinfo),
                         (int32_t *)(S + L.o_ntt), shared_tc ? (int)shT : 0,
                         (flags & HAR_CUDA_MOE_EMPTY_SLOTS) ? 1 : 0,
                         L.o_gcnt ? (int32_t *)(S + L.o_gcnt) : nullptr);
  if (st) return st;
  // tensor-core path parameters (experts with >= thr tokens)
  TcParams tp{};
  TcMaps gmaps{}, dmaps{};
  if (tc) {
    tp.E = E;
    tp.T = (int)T;
    tp.k = k;
    tp.n = (int)n;
    tp.shared_tc = shared_tc ? 1 : 0;
    tp.tt_info = (const int2 *)(S + L.o_ttinfo);
    tp.n_tt = (const int32_t *)(S + L.o_ntt);
    tp.a16 = (__half *)(S + L.o_a16);
    tp.ybuf = p.ybuf;
    tp.status = ctx->d_status;
    if (!layer->tc_maps)
      return set_error(ctx, HAR_CUDA_ERR_UNSUPPORTED, "moe_ffn: layer has no tensor-core maps");
    gmaps.a0 = layer->map_gate;
    gmaps.a1 = layer->map_up;
    dmaps.a0 = layer->map_down;
    dmaps.a1 = layer->map_down;
    if (has_sh) {
      gmaps.sh0 = layer->map_sh_gate;
      gmaps.sh1 = layer->map_sh_up;
      dmaps.sh0 = layer->map_sh_down;
      dmaps.sh1 = layer->map_sh_down;
    }
    // token rows in slot order (f16 hi/lo row pairs): the B operands, one box
    // of 32/64 rows x 64 values per K-step; and their min-term operands, two
    // boxes of 32/64 rows x 8 values per super-block
    const uint64_t rows2 = 2 * (uint64_t)(n + T);
    for (int bx = 0; bx < TC_NBOX; ++bx) {
      if ((st = encode_tmap_2d(ctx, &gmaps.s16[bx], S + L.o_xs16, 2, rows2, (uint64_t)(H / 16),
                               (uint64_t)(H / 16) * 2, 32u << bx, 8, false)))
        return st;
      if ((st = encode_tmap_2d(ctx, &dmaps.s16[bx], S + L.o_as16, 2, rows2, (uint64_t)(I / 16),
                               (uint64_t)(I / 16) * 2, 32u << bx, 8, false)))
        return st;
    }
    for (int bx = 0; bx < TC_NBOX; ++bx) {
      if ((st = encode_tmap_2d(ctx, &gmaps.b[bx], S + L.o_x16, 2, rows2, (uint64_t)H,
                               (uint64_t)H * 2, 32u << bx, 64, true)))
        return st;
      if ((st = encode_tmap_2d(ctx, &dmaps.b[bx], S + L.o_a16, 2, rows2, (uint64_t)I,
                               (uint64_t)I * 2, 32u << bx, 64, true)))
        return st;
    }
    if ((st = launch_gather_f16(ctx, x, H, p.order, ids, p.counts, p.offsets + E, thr, (int)n, k,
                                (int)sh0, (int)shT, tp.shared_tc, (__half *)(S + L.o_x16), (__half *)(S + L.o_xs16),
                                tp.shared_tc ? layer->sh_gate_inp : nullptr, (float *)(S + L.o_gsh))))
      return st;
  }
  if (gate_row && shT > 0 && !(tc && shared_tc)) {
    prof_begin(ctx);
    shared_gate_kernel<<<(unsigned)((shT + 7) / 8), 256, 0, ctx->stream>>>(layer->sh_gate_inp, x, H, (int)sh0,
                                                                          (int)shT, (float *)(S + L.o_gsh));
    if ((st = check_launch(ctx, "shared_gate_kernel"))) return st;
  }
  // upper bound of tensor-core token tiles: each big expert has >= thr tokens
  const int64_t max_tc_tt =
      tc ? std::min<int64_t>(E, n / std::max(thr, 1)) + n / TC_NT + 2 + (shared_tc ? shT / TC_NT + 1 : 0) : 0;
  if (q8 && (st = launch_q8k_quantize(ctx, x, T, H, S + o_xq))) return st;
  const int max_groups = (int)std::min<int64_t>(E, n) + p.has_shared;
  const int grid_cap = ctx->num_sms * 4;
  // the CUDA-core kernels have work unless every non-empty expert (threshold 1)
  // and the shared expert take the tensor-core path
  const bool gemv_work = !tc || thr > 1 || p.gemv_shared;
  if (gemv_work) {
    const int rpt = rows_per_tile_gu(H), ntg = (I + rpt - 1) / rpt;
    const int grid = std::max(1, std::min(grid_cap, max_groups * ntg));
    st = q8 ? dispatch_gate_up<ACT_Q8K>(ctx, p, grid) : dispatch_gate_up<ACT_F32>(ctx, p, grid);
    if (st) return st;
  }
  if (tc) {
    TcParams g = tp;
    g.rows = I;
    g.K = H;
    g.out_ld = I;
    g.w0 = p.gate;
    g.w1 = p.up;
    g.sw0 = p.sh_gate;
    g.sw1 = p.sh_up;
    g.row_bytes = p.rb_h;
    g.s16_out = (__half *)(S + L.o_as16);
    st = f16w ? launch_moe_tc_f16w(ctx, gmaps, g, 2, (int)std::min<int64_t>(INT_MAX, max_tc_tt * (I / TC_M)))
              : launch_moe_tc(ctx, gmaps, g, 2, (int)std::min<int64_t>(INT_MAX, max_tc_tt * (I / TC_M)));
    if (st) return st;
  }
  if (q8 && (st = launch_q8k_quantize(ctx, p.a, n + (p.has_shared ? shT : 0), I, S + o_aq))) return st;
  if (gemv_work) {
    const int rpt = rows_per_tile_d(I), ntg = (H + rpt - 1) / rpt;
    const int grid = std::max(1, std::min(grid_cap, max_groups * ntg));
    st = q8 ? dispatch_down<ACT_Q8K>(ctx, p, grid) : dispatch_down<ACT_F32>(ctx, p, grid);
    if (st) return st;
  }
  if (tc) {
    TcParams d = tp;
    d.rows = H;
    d.K = I;
    d.out_ld = H;
    d.w0 = d.w1 = p.down;
    d.sw0 = d.sw1 = p.sh_down;
    d.row_bytes = p.rb_i;
    d.s16_out = nullptr;
    st = f16w ? launch_moe_tc_f16w(ctx, dmaps, d, 1, (int)std::min<int64_t>(INT_MAX, max_tc_tt * (H / TC_M)))
              : launch_moe_tc(ctx, dmaps, d, 1, (int)std::min<int64_t>(INT_MAX, max_tc_tt * (H / TC_M)));
    if (st) return st;
  }
  prof_begin(ctx);
  moe_combine_kernel<<<dim3((unsigned)T, (unsigned)((H / 4 + COMB_T - 1) / COMB_T)), COMB_T, 0, ctx->stream>>>(
      p, x, weights, y, (flags & HAR_CUDA_MOE_ADD_RESIDUAL) ? 1 : 0);
  return check_launch(ctx, "moe_combine_kernel");
}

}  // namespace har
