// k_route.cu — router softmax + top-k, and the stable expert-major grouping.
//
// route_topk_kernel restates routed_moe's selection
// (har/crates/har-demo/src/bin/har-native-qwen35moe.rs:1167-1204) with the
// reference's f32 operation order: max fold, exp(l - max), sequential sum in
// index order clamped to >= 1e-9, p = e / sum, order by p descending then
// lower index, take k, renormalise by the sequential sum of the selected p
// (clamped to >= 1e-9).  exp is expf_ref, the reference's f32::exp (glibc's
// expf) restated, so ids and weights are bit-exact.
//
// group_kernel restates MoEModel::forward_batch's grouping
// (har/crates/har-serve/src/moe.rs:195-202): groups[e] holds the entries
// (t*k + slot) routed to e in position order.  It is a stable counting sort
// in one CTA of 16 warps (E <= 2048): each warp owns a contiguous segment of entries,
// counts per expert with __match_any_sync, a scan turns counts into offsets,
// and a second pass writes positions.
#include "har_internal.cuh"
#include "tc_ptx.cuh"

namespace har {

// ---------------------------------------------------------------------------
// route_topk: one warp per token; the warp's exps live in shared memory.
// ---------------------------------------------------------------------------
// One token's selection by one warp: l its E logits (read through L2, so a
// warp may read logits other CTAs of the same kernel wrote), p E floats of
// shared memory (16-byte aligned when E % 4 == 0), results to ids[0..k) and
// weights[0..k).
__device__ __forceinline__ void topk_warp(const float *l, int E, int k, float *p, int lane,
                                          int32_t *ids, float *weights) {
  float mx = -INFINITY;
  for (int i = lane; i < E; i += 32) mx = fmaxf(mx, __ldcg(l + i));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
#pragma unroll 4
  for (int i = lane; i < E; i += 32) p[i] = expf_ref(__fsub_rn(__ldcg(l + i), mx));
  __syncwarp();
  float den = 0.0f;
  if (lane == 0) {  // exps.iter().sum(): one chain in index order
    int i = 0;
    if (E % 4 == 0) {  // the warp's row is then 16-byte aligned: four values per load
      const float4 *p4 = reinterpret_cast<const float4 *>(p);
#pragma unroll 8
      for (; i < E; i += 4) {
        const float4 v = p4[i >> 2];
        den = __fadd_rn(den, v.x);
        den = __fadd_rn(den, v.y);
        den = __fadd_rn(den, v.z);
        den = __fadd_rn(den, v.w);
      }
    }
    for (; i < E; ++i) den = __fadd_rn(den, p[i]);
    den = fmaxf(den, ROUTER_EPS);
  }
  den = __shfl_sync(0xffffffffu, den, 0);
#pragma unroll 4
  for (int i = lane; i < E; i += 32) p[i] = __fdiv_rn(p[i], den);
  __syncwarp();
  // k rounds of warp arg-max over (p desc, index asc).  Every p is >= +0, so
  // its bits order like its value (and a positive NaN above +inf, as
  // total_cmp orders it); selected entries are marked by their sign bit.
  // Each lane's best (scanned in index order, strict >: the lowest index of
  // a tie) goes into one warp max of the bits and one warp min of the index
  // among the lanes holding that max.
  int sel_id = 0;
  float sel_p = 0.0f;
  for (int s = 0; s < k; ++s) {
    uint32_t bb = 0;
    int bi = 0x7fffffff;
    for (int i = lane; i < E; i += 32) {
      const uint32_t v = __float_as_uint(p[i]);
      if (v < 0x80000000u && (v > bb || bi == 0x7fffffff)) {
        bb = v;
        bi = i;
      }
    }
    const uint32_t mb = __reduce_max_sync(0xffffffffu, bb);
    const int wi = (int)__reduce_min_sync(0xffffffffu, bb == mb ? (uint32_t)bi : 0x7fffffffu);
    if (lane == s) {
      sel_id = wi;
      sel_p = __uint_as_float(mb);
    }
    if (lane == 0) p[wi] = __uint_as_float(mb | 0x80000000u);
    __syncwarp();
  }
  float tot = 0.0f;
  for (int s = 0; s < k; ++s) tot = __fadd_rn(tot, __shfl_sync(0xffffffffu, sel_p, s));
  tot = fmaxf(tot, ROUTER_EPS);
  if (lane < k) {
    ids[lane] = sel_id;
    weights[lane] = __fdiv_rn(sel_p, tot);
  }
}

// topk_warp with the token's values held in registers: lane l owns indices
// l, l + 32, ... (EPL of them, E <= 32 * EPL).  The logits are read in one
// burst, the exps are staged in p only for the sequential sum, and each of the
// k rounds is an in-register tournament (lower index wins a tie, as the scan in
// index order does) plus two warp reductions.  Same operations in the same
// order as topk_warp, so the same bits.
// One level of the in-register tournament (entries W apart), then the next.
template <int EPL, int W>
__device__ __forceinline__ void topk_tournament(uint32_t (&bk)[EPL], int (&bj)[EPL]) {
  if constexpr (W < EPL) {
#pragma unroll
    for (int j = 0; j + W < EPL; j += 2 * W) {
      const bool la = bk[j] < 0x80000000u, ra = bk[j + W] < 0x80000000u;
      if (ra && (!la || bk[j + W] > bk[j])) {
        bk[j] = bk[j + W];
        bj[j] = bj[j + W];
      }
    }
    topk_tournament<EPL, 2 * W>(bk, bj);
  }
}

template <int EPL>
__device__ __forceinline__ void topk_warp_regs(const float *l, int E, int k, float *p, int lane,
                                               int32_t *ids, float *weights) {
  float v[EPL];
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int i = lane + 32 * j;
    v[j] = i < E ? __ldcg(l + i) : -INFINITY;
  }
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < EPL; ++j) mx = fmaxf(mx, v[j]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int i = lane + 32 * j;
    v[j] = expf_ref(__fsub_rn(v[j], mx));
    if (i < E) p[i] = v[j];
  }
  __syncwarp();
  float den = 0.0f;
  if (lane == 0) {  // exps.iter().sum(): one chain in index order
    int i = 0;
    if (E % 4 == 0) {
      const float4 *p4 = reinterpret_cast<const float4 *>(p);
#pragma unroll 8
      for (; i < E; i += 4) {
        const float4 q = p4[i >> 2];
        den = __fadd_rn(den, q.x);
        den = __fadd_rn(den, q.y);
        den = __fadd_rn(den, q.z);
        den = __fadd_rn(den, q.w);
      }
    }
    for (; i < E; ++i) den = __fadd_rn(den, p[i]);
    den = fmaxf(den, ROUTER_EPS);
  }
  den = __shfl_sync(0xffffffffu, den, 0);
  // keys: the bits of p (>= +0, ordered like the values); taken entries and
  // padding have the sign bit set
  uint32_t key[EPL];
#pragma unroll
  for (int j = 0; j < EPL; ++j)
    key[j] = lane + 32 * j < E ? __float_as_uint(__fdiv_rn(v[j], den)) : 0xffffffffu;
  int sel_id = 0;
  float sel_p = 0.0f;
  for (int s = 0; s < k; ++s) {
    // this lane's best available entry: a tournament over j, left (lower j,
    // lower index) kept unless the right one is available and larger
    uint32_t bk[EPL];
    int bj[EPL];
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
      bk[j] = key[j];
      bj[j] = j;
    }
    topk_tournament<EPL, 1>(bk, bj);
    const bool avail = bk[0] < 0x80000000u;
    const uint32_t bb = avail ? bk[0] : 0u;
    const uint32_t bi = avail ? (uint32_t)(lane + 32 * bj[0]) : 0x7fffffffu;
    const uint32_t mb = __reduce_max_sync(0xffffffffu, bb);
    const uint32_t wi = __reduce_min_sync(0xffffffffu, bb == mb ? bi : 0x7fffffffu);
    if (lane == s) {
      sel_id = (int)wi;
      sel_p = __uint_as_float(mb);
    }
    // mark the winner taken (branch-free: an indexed register write would
    // put the keys in local memory)
    const uint32_t hit = wi != 0x7fffffffu && lane == (int)(wi & 31u) ? 0x80000000u : 0u;
    const int jw = (int)(wi >> 5);
#pragma unroll
    for (int j = 0; j < EPL; ++j) key[j] |= j == jw ? hit : 0u;
  }
  float tot = 0.0f;
  for (int s = 0; s < k; ++s) tot = __fadd_rn(tot, __shfl_sync(0xffffffffu, sel_p, s));
  tot = fmaxf(tot, ROUTER_EPS);
  if (lane < k) {
    ids[lane] = sel_id;
    weights[lane] = __fdiv_rn(sel_p, tot);
  }
  __syncwarp();  // p is reused by the warp's next token
}

// One token's selection by one warp, in registers when E <= 1024.
__device__ __forceinline__ void topk_token(const float *l, int E, int k, float *p, int lane, int32_t *ids,
                                           float *weights) {
  if (E <= 32) topk_warp_regs<1>(l, E, k, p, lane, ids, weights);
  else if (E <= 64) topk_warp_regs<2>(l, E, k, p, lane, ids, weights);
  else if (E <= 128) topk_warp_regs<4>(l, E, k, p, lane, ids, weights);
  else if (E <= 256) topk_warp_regs<8>(l, E, k, p, lane, ids, weights);
  else if (E <= 512) topk_warp_regs<16>(l, E, k, p, lane, ids, weights);
  else if (E <= 1024) topk_warp_regs<32>(l, E, k, p, lane, ids, weights);
  else topk_warp(l, E, k, p, lane, ids, weights);
}

// One token's selection by a whole CTA of TK_W warps, for the latency of a
// single token: thread th owns indices th, th + 32*TK_W, ... (EPT of them,
// E <= 32*TK_W*EPT), so the exps and divisions are spread 4x thinner than in
// topk_warp_regs.  Each warp takes its own k best (its entries in the same
// (p desc, index asc) order), and the k best of the union are found by rank:
// an entry's rank is the number of candidates ahead of it in that order.  The
// global k best are all among their warps' k best, so the result is the
// reference's.  p: E floats of shared memory.
constexpr int TK_W = 4, TK_T = 32 * TK_W;

struct TopkCtaSmem {
  float red[TK_W + 1];
  uint32_t ckey[TK_W * 32];
  int32_t cidx[TK_W * 32];
  int32_t out_id[32];
  float out_p[32];
};

template <int EPT>
__device__ __forceinline__ void topk_cta(const float *l, int E, int k, float *p, TopkCtaSmem &sm,
                                         int32_t *ids, float *weights) {
  const int th = threadIdx.x, warp = th >> 5, lane = th & 31;
  float v[EPT];
#pragma unroll
  for (int j = 0; j < EPT; ++j) {
    const int i = th + TK_T * j;
    v[j] = i < E ? __ldcg(l + i) : -INFINITY;
  }
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < EPT; ++j) mx = fmaxf(mx, v[j]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) sm.red[warp] = mx;
  __syncthreads();
#pragma unroll
  for (int w = 0; w < TK_W; ++w) mx = fmaxf(mx, sm.red[w]);
#pragma unroll
  for (int j = 0; j < EPT; ++j) {
    const int i = th + TK_T * j;
    v[j] = expf_ref(__fsub_rn(v[j], mx));
    if (i < E) p[i] = v[j];
  }
  __syncthreads();
  if (th == 0) {  // exps.iter().sum(): one chain in index order
    float den = 0.0f;
    int i = 0;
    if (E % 4 == 0) {
      const float4 *p4 = reinterpret_cast<const float4 *>(p);
#pragma unroll 8
      for (; i < E; i += 4) {
        const float4 q = p4[i >> 2];
        den = __fadd_rn(den, q.x);
        den = __fadd_rn(den, q.y);
        den = __fadd_rn(den, q.z);
        den = __fadd_rn(den, q.w);
      }
    }
    for (; i < E; ++i) den = __fadd_rn(den, p[i]);
    sm.red[TK_W] = fmaxf(den, ROUTER_EPS);
  }
  __syncthreads();
  const float den = sm.red[TK_W];
  uint32_t key[EPT];
#pragma unroll
  for (int j = 0; j < EPT; ++j)
    key[j] = th + TK_T * j < E ? __float_as_uint(__fdiv_rn(v[j], den)) : 0xffffffffu;
  // this warp's k best, in order, to the candidate list
  for (int s = 0; s < k; ++s) {
    uint32_t bk[EPT];
    int bj[EPT];
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
      bk[j] = key[j];
      bj[j] = j;
    }
    topk_tournament<EPT, 1>(bk, bj);
    const bool avail = bk[0] < 0x80000000u;
    const uint32_t bb = avail ? bk[0] : 0u;
    const uint32_t bi = avail ? (uint32_t)(th + TK_T * bj[0]) : 0x7fffffffu;
    const uint32_t mb = __reduce_max_sync(0xffffffffu, bb);
    const uint32_t wi = __reduce_min_sync(0xffffffffu, bb == mb ? bi : 0x7fffffffu);
    if (lane == 0) {
      sm.ckey[warp * k + s] = mb;
      sm.cidx[warp * k + s] = (int32_t)wi;  // 0x7fffffff: nothing left in this warp
    }
    const uint32_t hit = wi != 0x7fffffffu && (int)((wi % TK_T) >> 5) == warp && lane == (int)(wi & 31u)
                             ? 0x80000000u : 0u;
    const int jw = (int)(wi / TK_T);
#pragma unroll
    for (int j = 0; j < EPT; ++j) key[j] |= j == jw ? hit : 0u;
  }
  if (th < k) {  // slots past the available entries, as the round-by-round scan leaves them
    sm.out_id[th] = 0x7fffffff;
    sm.out_p[th] = 0.0f;
  }
  __syncthreads();
  const int nc = TK_W * k;
  if (th < nc && sm.cidx[th] != 0x7fffffff) {
    const uint32_t mk = sm.ckey[th];
    const int32_t mi = sm.cidx[th];
    int rank = 0;
#pragma unroll 8
    for (int c = 0; c < nc; ++c) {
      const int32_t ci = sm.cidx[c];
      const uint32_t ck = sm.ckey[c];
      rank += ci != 0x7fffffff && (ck > mk || (ck == mk && ci < mi));
    }
    if (rank < k) {
      sm.out_id[rank] = mi;
      sm.out_p[rank] = __uint_as_float(mk);
    }
  }
  __syncthreads();
  if (warp == 0) {
    const float sel_p = lane < k ? sm.out_p[lane] : 0.0f;
    float tot = 0.0f;
    for (int s = 0; s < k; ++s) tot = __fadd_rn(tot, __shfl_sync(0xffffffffu, sel_p, s));
    tot = fmaxf(tot, ROUTER_EPS);
    if (lane < k) {
      ids[lane] = sm.out_id[lane];
      weights[lane] = __fdiv_rn(sel_p, tot);
    }
  }
}

// The CTA-wide selection for E <= 1024; false when E is larger.
__device__ __forceinline__ bool topk_cta_token(const float *l, int E, int k, float *p, TopkCtaSmem &sm,
                                               int32_t *ids, float *weights) {
  if (E <= TK_T) topk_cta<1>(l, E, k, p, sm, ids, weights);
  else if (E <= 2 * TK_T) topk_cta<2>(l, E, k, p, sm, ids, weights);
  else if (E <= 4 * TK_T) topk_cta<4>(l, E, k, p, sm, ids, weights);
  else if (E <= 8 * TK_T) topk_cta<8>(l, E, k, p, sm, ids, weights);
  else return false;
  return true;
}

// One CTA per token (small T: the tokens' selections run side by side).
__global__ void __launch_bounds__(TK_T) route_topk_cta_kernel(const float *__restrict__ logits, int E, int k,
                                                              int32_t *__restrict__ ids,
                                                              float *__restrict__ weights) {
  extern __shared__ __align__(16) float tks[];
  __shared__ TopkCtaSmem sm;
  const int64_t t = blockIdx.x;
  pdl_wait();
  pdl_launch_dependents();
  topk_cta_token(logits + t * E, E, k, tks, sm, ids + t * k, weights + t * k);
}

__global__ void __launch_bounds__(128, 1) route_topk_kernel(const float *__restrict__ logits,
                                                         int64_t T, int E, int k,
                                                         int32_t *__restrict__ ids,
                                                         float *__restrict__ weights) {
  extern __shared__ float rsm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * 4 + warp;
  if (t >= T) return;
  topk_token(logits + t * E, E, k, rsm + (size_t)warp * E, lane, ids + t * k, weights + t * k);
}

// tokens per call up to which each token gets a CTA of its own
constexpr int64_t TK_CTA_MAX_T = 64;

int32_t launch_route_topk(har_cuda_ctx *ctx, const float *logits, int64_t T, int E, int k,
                          int32_t *ids, float *weights) {
  if (T <= TK_CTA_MAX_T && E <= 8 * TK_T) {
    prof_begin(ctx);
    launch_pdl(route_topk_cta_kernel, dim3((unsigned)T), dim3(TK_T), sizeof(float) * (size_t)E, ctx->stream,
               logits, E, k, ids, weights);
    return check_launch(ctx, "route_topk_cta_kernel");
  }
  const size_t smem = (size_t)4 * E * sizeof(float);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(route_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int64_t grid = (T + 3) / 4;
  prof_begin(ctx);
  route_topk_kernel<<<(unsigned)grid, 128, smem, ctx->stream>>>(logits, T, E, k, ids, weights);
  return check_launch(ctx, "route_topk_kernel");
}

// ---------------------------------------------------------------------------
// Grouping: a stable counting sort of n = T*k entries by expert id
// (MoEModel::forward_batch's groups, har/crates/har-serve/src/moe.rs:195-202).
// Outputs counts[E], offsets[E+1], order[n] (entry at each grouped position),
// inv[n] (grouped position of each entry) and, when ne != null, the list of
// non-empty experts in expert order (ne[0..*n_ne)) below `thr` tokens, and
// the token tiles of the experts at or above it (group_lists).  Entries with
// an out-of-range id set DEV_ERR_BOUNDS in *status and are dropped; with
// allow_empty, id -1 marks an empty slot and is dropped silently.
//
// Within a CTA of GROUP_WARPS warps each warp owns a contiguous run of
// entries, counts them per expert with __match_any_sync (pass 1), and after a
// scan places them (pass 2) — stable because runs, and entries within a run,
// keep their order.  Up to GROUP_MC_MIN entries one CTA does everything
// (group_kernel).  Above it the entries are cut into contiguous segments, one
// CTA each: group_count_kernel counts a segment per expert, group_scan_kernel
// (one CTA) turns the segments' counts into per-segment bases, the offsets and
// the lists, and group_scatter_kernel recounts its segment per warp and
// places it.  Measured on B200 in a CUDA graph: one CTA takes ~40 us for
// 20,480 entries (the local layer of an 8-way expert-parallel step) and
// ~21 us for 8,192; the three launches take ~10 and ~10 us (~13 us at 40,960).
// ---------------------------------------------------------------------------
constexpr int GROUP_WARPS = 16;
constexpr int64_t GROUP_MC_MIN = 2048;  // entries above which the CTAs share the sort
constexpr int GROUP_SEG = 1024;         // entries per segment (64 per warp)
constexpr int GROUP_MAX_SEGS = 512;

__host__ __device__ inline int group_segments(int64_t n) {
  if (n <= GROUP_MC_MIN) return 1;
  const int64_t s = (n + GROUP_SEG - 1) / GROUP_SEG;
  return (int)(s < GROUP_MAX_SEGS ? s : GROUP_MAX_SEGS);
}

// Pass 1 for one warp: cnt[e] += entries of [s0, s1) with id e.  Ids are
// loaded GB chunks of 32 at a time before the warp-synchronous updates, so one
// load latency covers 32 * GB entries.  status != null reports bad ids.
constexpr int GB = 8;
__device__ __forceinline__ void group_count_run(const int32_t *ids, int s0, int s1, int E, int32_t *cnt,
                                                int allow_empty, int *status, int lane) {
  const unsigned lt = (1u << lane) - 1u;
  for (int b0 = s0; b0 < s1; b0 += 32 * GB) {
    int ev[GB];
#pragma unroll
    for (int j = 0; j < GB; ++j) {
      const int i = b0 + 32 * j + lane;
      ev[j] = i < s1 ? ids[i] : -1;
    }
#pragma unroll
    for (int j = 0; j < GB; ++j) {
      const int i = b0 + 32 * j + lane;
      int e = ev[j];
      if (i < s1 && (e < 0 || e >= E)) {
        if (status && !(allow_empty && e == -1)) atomicOr(status, DEV_ERR_BOUNDS);
        e = -1;
      }
      const unsigned m = __match_any_sync(0xffffffffu, e);
      if (e >= 0 && (m & lt) == 0) cnt[e] += __popc(m);
      __syncwarp();
    }
  }
}

// Pass 2 for one warp: entries of [s0, s1) to their positions; base[e] is
// where this warp's next entry of expert e goes (advanced as it places).
__device__ __forceinline__ void group_place_run(const int32_t *ids, int s0, int s1, int E, int32_t *base,
                                                int32_t *order, int32_t *inv, int lane) {
  const unsigned lt = (1u << lane) - 1u;
  for (int b0 = s0; b0 < s1; b0 += 32 * GB) {
    int ev[GB];
#pragma unroll
    for (int j = 0; j < GB; ++j) {
      const int i = b0 + 32 * j + lane;
      ev[j] = i < s1 ? ids[i] : -1;
    }
#pragma unroll
    for (int j = 0; j < GB; ++j) {
      const int i = b0 + 32 * j + lane;
      int e = ev[j];
      if (e < 0 || e >= E) e = -1;
      const unsigned m = __match_any_sync(0xffffffffu, e);
      int pos = 0;
      if (e >= 0) pos = base[e] + __popc(m & lt);
      __syncwarp();
      if (e >= 0) {
        order[pos] = i;
        inv[i] = pos;
        if ((m & lt) == 0) base[e] += __popc(m);
      } else if (i < s1) {
        inv[i] = -1;
      }
      __syncwarp();
    }
  }
}

// The run of warp w of GROUP_WARPS over [c0, c1).
__device__ __forceinline__ void group_run(int c0, int c1, int w, int &s0, int &s1) {
  const int seg = (c1 - c0 + GROUP_WARPS - 1) / GROUP_WARPS;
  s0 = min(c1, c0 + w * seg);
  s1 = min(c1, s0 + seg);
}

// Per-warp counts cnt[w][e] become each warp's base within expert e (plus
// add[e] when given); tot[e] = the CTA's count of e.  Block-wide.
__device__ __forceinline__ void group_warp_bases(int32_t *cnt, int E, const int32_t *add, int32_t *tot) {
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = add ? add[e] : 0;
    for (int w = 0; w < GROUP_WARPS; ++w) {
      const int c = cnt[w * E + e];
      cnt[w * E + e] = run;
      run += c;
    }
    if (tot) tot[e] = run - (add ? add[e] : 0);
  }
}

// off[0..E] = exclusive scan of tot[0..E) (off[E] = the total), block-wide,
// in chunks of blockDim; warp_tot holds GROUP_WARPS + 1 words of scratch.
__device__ __forceinline__ void group_offsets(const int32_t *tot, int E, int32_t *off, int32_t *warp_tot) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int base = 0; base < E; base += blockDim.x) {
    const int e = base + threadIdx.x;
    const int t = e < E ? tot[e] : 0;
    int v = t;  // inclusive warp scan
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += u;
    }
    if (lane == 31) warp_tot[warp] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
      int r = base == 0 ? 0 : off[base];
      for (int w = 0; w < GROUP_WARPS; ++w) {
        const int x = warp_tot[w];
        warp_tot[w] = r;
        r += x;
      }
      warp_tot[GROUP_WARPS] = r;
    }
    __syncthreads();
    if (e < E) off[e] = warp_tot[warp] + v - t;
    if (threadIdx.x == 0) off[min(E, base + (int)blockDim.x)] = warp_tot[GROUP_WARPS];
    __syncthreads();
  }
}

// Non-empty experts in expert order, split by token count: ne[] those below
// `thr` (CUDA-core path); those at or above it (tensor-core path) are cut
// into ceil(count/nt) token tiles, listed in expert order as
// tt_info[j] = {expert | tokens << 16, first slot}.  When shared_T > 0 the
// shared expert (index E, slots n .. n + shared_T) follows with
// ceil(shared_T/nt) tiles.  *n_ne / *n_tt = the list lengths.  Each warp takes
// chunks of 32 experts; a scan of the chunks' totals (in `scratch`, 2 words
// per chunk) gives each chunk its offsets.  Block-wide; off[] in shared memory.
__device__ __forceinline__ void group_lists(const int32_t *off, int E, int n, int thr, int nt,
                                            int32_t *ne, int32_t *n_ne, int2 *tt_info, int32_t *n_tt,
                                            int shared_T, int32_t *scratch, int32_t *warp_tot) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned lt = (1u << lane) - 1u;
  const int nch = (E + 31) / 32;
  int32_t *ch_small = scratch, *ch_tt = scratch + nch;
  __syncthreads();
  for (int c = warp; c < nch; c += GROUP_WARPS) {
    const int e = c * 32 + lane;
    const int ce = e < E ? off[e + 1] - off[e] : 0;
    const bool small = ce > 0 && ce < thr;
    const int tt = ce > 0 && ce >= thr ? (ce + nt - 1) / nt : 0;
    const int ns = __popc(__ballot_sync(0xffffffffu, small));
    const int ntt = __reduce_add_sync(0xffffffffu, (unsigned)tt);
    if (lane == 0) {
      ch_small[c] = ns;
      ch_tt[c] = ntt;
    }
  }
  __syncthreads();
  if (warp == 0) {  // exclusive scans over the chunks
    int rs = 0, rt = 0;
    for (int base = 0; base < nch; base += 32) {
      const int c = base + lane;
      const int a = c < nch ? ch_small[c] : 0, b = c < nch ? ch_tt[c] : 0;
      int ia = a, ib = b;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int ua = __shfl_up_sync(0xffffffffu, ia, o), ub = __shfl_up_sync(0xffffffffu, ib, o);
        if (lane >= o) {
          ia += ua;
          ib += ub;
        }
      }
      if (c < nch) {
        ch_small[c] = rs + ia - a;
        ch_tt[c] = rt + ib - b;
      }
      rs += __shfl_sync(0xffffffffu, ia, 31);
      rt += __shfl_sync(0xffffffffu, ib, 31);
    }
    if (lane == 0) {
      *n_ne = rs;
      *n_tt = rt + (shared_T + nt - 1) / nt;
      warp_tot[0] = rt;  // first tile of the shared expert
    }
  }
  __syncthreads();
  for (int c = warp; c < nch; c += GROUP_WARPS) {
    const int e = c * 32 + lane;
    const int ce = e < E ? off[e + 1] - off[e] : 0;
    const bool small = ce > 0 && ce < thr;
    const int tt = ce > 0 && ce >= thr ? (ce + nt - 1) / nt : 0;
    const unsigned bm = __ballot_sync(0xffffffffu, small);
    if (small) ne[ch_small[c] + __popc(bm & lt)] = e;
    int incl = tt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += u;
    }
    for (int j = 0; j < tt; ++j)
      tt_info[ch_tt[c] + incl - tt + j] = make_int2(e | (min(nt, ce - j * nt) << 16), off[e] + j * nt);
  }
  const int run_tt = warp_tot[0];
  for (int t0 = (int)threadIdx.x * nt; t0 < shared_T; t0 += (int)blockDim.x * nt)
    tt_info[run_tt + t0 / nt] = make_int2(E | (min(nt, shared_T - t0) << 16), n + t0);
}

// One CTA: the whole sort.
__global__ void __launch_bounds__(GROUP_WARPS * 32) group_kernel(
    const int32_t *__restrict__ ids, int n, int E, int32_t *__restrict__ counts,
    int32_t *__restrict__ offsets, int32_t *__restrict__ order, int32_t *__restrict__ inv,
    int32_t *__restrict__ ne, int32_t *__restrict__ n_ne, int thr, int nt,
    int2 *__restrict__ tt_info, int32_t *__restrict__ n_tt, int shared_T, int allow_empty,
    int *status) {
  extern __shared__ __align__(16) uint8_t gsm[];
  int32_t *cnt = reinterpret_cast<int32_t *>(gsm);  // [W][E]
  int32_t *off = cnt + (size_t)GROUP_WARPS * E;      // [E+1]
  int32_t *tot = off + E + 1;                         // [E]
  __shared__ int32_t warp_tot[GROUP_WARPS + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < GROUP_WARPS * E; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  int s0, s1;
  group_run(0, n, warp, s0, s1);
  group_count_run(ids, s0, s1, E, cnt + warp * E, allow_empty, status, lane);
  __syncthreads();
  group_warp_bases(cnt, E, nullptr, tot);
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) counts[e] = tot[e];
  group_offsets(tot, E, off, warp_tot);
  for (int e = threadIdx.x; e <= E; e += blockDim.x) offsets[e] = off[e];
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int o = off[e];
    for (int w = 0; w < GROUP_WARPS; ++w) cnt[w * E + e] += o;
  }
  __syncthreads();
  group_place_run(ids, s0, s1, E, cnt + warp * E, order, inv, lane);
  if (ne) group_lists(off, E, n, thr, nt, ne, n_ne, tt_info, n_tt, shared_T, cnt, warp_tot);
}

// Several CTAs, 1 of 3: segment b's count of every expert, gcnt[b][e].
__global__ void __launch_bounds__(GROUP_WARPS * 32) group_count_kernel(
    const int32_t *__restrict__ ids, int n, int E, int seg, int32_t *__restrict__ gcnt, int allow_empty,
    int *status) {
  extern __shared__ __align__(16) uint8_t gsm[];
  int32_t *cnt = reinterpret_cast<int32_t *>(gsm);  // [W][E]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < GROUP_WARPS * E; i += blockDim.x) cnt[i] = 0;
  pdl_wait();  // the ids come from the previous launch
  pdl_launch_dependents();
  __syncthreads();
  const int c0 = min(n, (int)blockIdx.x * seg), c1 = min(n, c0 + seg);
  int s0, s1;
  group_run(c0, c1, warp, s0, s1);
  group_count_run(ids, s0, s1, E, cnt + warp * E, allow_empty, status, lane);
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int t = 0;
    for (int w = 0; w < GROUP_WARPS; ++w) t += cnt[w * E + e];
    gcnt[(size_t)blockIdx.x * E + e] = t;
  }
}

// 2 of 3 (one CTA): gcnt[b][e] becomes segment b's first position within
// expert e; the counts, offsets and lists as in group_kernel.
__global__ void __launch_bounds__(GROUP_WARPS * 32) group_scan_kernel(
    int32_t *__restrict__ gcnt, int B, int n, int E, int32_t *__restrict__ counts,
    int32_t *__restrict__ offsets, int32_t *__restrict__ ne, int32_t *__restrict__ n_ne, int thr, int nt,
    int2 *__restrict__ tt_info, int32_t *__restrict__ n_tt, int shared_T) {
  extern __shared__ __align__(16) uint8_t gsm[];
  int32_t *off = reinterpret_cast<int32_t *>(gsm);  // [E+1]
  int32_t *tot = off + E + 1;                        // [E]
  int32_t *scratch = tot + E;                        // [2 * ceil(E/32)]
  __shared__ int32_t warp_tot[GROUP_WARPS + 1];
  pdl_wait();
  pdl_launch_dependents();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = 0;
    for (int b = 0; b < B; ++b) {
      const int c = gcnt[(size_t)b * E + e];
      gcnt[(size_t)b * E + e] = run;
      run += c;
    }
    tot[e] = run;
    counts[e] = run;
  }
  __syncthreads();
  group_offsets(tot, E, off, warp_tot);
  for (int e = threadIdx.x; e <= E; e += blockDim.x) offsets[e] = off[e];
  if (ne) group_lists(off, E, n, thr, nt, ne, n_ne, tt_info, n_tt, shared_T, scratch, warp_tot);
}

// 3 of 3: segment b's entries to offsets[e] + gcnt[b][e] + their rank in it.
__global__ void __launch_bounds__(GROUP_WARPS * 32) group_scatter_kernel(
    const int32_t *__restrict__ ids, int n, int E, int seg, const int32_t *__restrict__ gcnt,
    const int32_t *__restrict__ offsets, int32_t *__restrict__ order, int32_t *__restrict__ inv) {
  extern __shared__ __align__(16) uint8_t gsm[];
  int32_t *cnt = reinterpret_cast<int32_t *>(gsm);  // [W][E]
  int32_t *add = cnt + (size_t)GROUP_WARPS * E;      // [E]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < GROUP_WARPS * E; i += blockDim.x) cnt[i] = 0;
  pdl_wait();
  pdl_launch_dependents();
  for (int e = threadIdx.x; e < E; e += blockDim.x) add[e] = offsets[e] + gcnt[(size_t)blockIdx.x * E + e];
  __syncthreads();
  const int c0 = min(n, (int)blockIdx.x * seg), c1 = min(n, c0 + seg);
  int s0, s1;
  group_run(c0, c1, warp, s0, s1);
  group_count_run(ids, s0, s1, E, cnt + warp * E, 1, nullptr, lane);
  __syncthreads();
  group_warp_bases(cnt, E, add, nullptr);
  __syncthreads();
  group_place_run(ids, s0, s1, E, cnt + warp * E, order, inv, lane);
}

size_t group_smem_bytes(int E) {
  return ((size_t)GROUP_WARPS * E + 2 * (size_t)E + 1) * 4;
}

// Scratch words the multi-CTA sort needs beside the outputs (0: one CTA).
size_t group_scratch_words(int64_t n, int E) {
  const int B = group_segments(n);
  return B > 1 ? (size_t)B * E : 0;
}

int32_t launch_group_full(har_cuda_ctx *ctx, const int32_t *ids, int64_t n, int E,
                          int32_t *counts, int32_t *offsets, int32_t *order, int32_t *inv,
                          int32_t *ne, int32_t *n_ne, int thr, int nt, int2 *tt_info,
                          int32_t *n_tt, int shared_T, int allow_empty, int32_t *gcnt) {
  const size_t smem = group_smem_bytes(E);
  const int B = group_segments(n);
  if (B == 1 || !gcnt) {
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(group_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    prof_begin(ctx);
    group_kernel<<<1, GROUP_WARPS * 32, smem, ctx->stream>>>(ids, (int)n, E, counts, offsets, order, inv,
                                                             ne, n_ne, thr, nt, tt_info, n_tt, shared_T,
                                                             allow_empty, ctx->d_status);
    return check_launch(ctx, "group_kernel");
  }
  const int seg = (int)((n + B - 1) / B);
  if (smem > 48 * 1024) {
    cudaFuncSetAttribute(group_count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaFuncSetAttribute(group_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaFuncSetAttribute(group_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  }
  prof_begin(ctx);
  launch_pdl(group_count_kernel, dim3(B), dim3(GROUP_WARPS * 32), smem, ctx->stream, ids, (int)n, E, seg,
             gcnt, allow_empty, ctx->d_status);
  int32_t st = check_launch(ctx, "group_count_kernel");
  if (st) return st;
  prof_begin(ctx);
  launch_pdl(group_scan_kernel, dim3(1), dim3(GROUP_WARPS * 32), smem, ctx->stream, gcnt, B, (int)n, E,
             counts, offsets, ne, n_ne, thr, nt, tt_info, n_tt, shared_T);
  if ((st = check_launch(ctx, "group_scan_kernel"))) return st;
  prof_begin(ctx);
  launch_pdl(group_scatter_kernel, dim3(B), dim3(GROUP_WARPS * 32), smem, ctx->stream, ids, (int)n, E, seg,
             (const int32_t *)gcnt, (const int32_t *)offsets, order, inv);
  return check_launch(ctx, "group_scatter_kernel");
}

int32_t launch_group(har_cuda_ctx *ctx, const int32_t *ids, int64_t T, int k, int E,
                     int32_t *counts, int32_t *offsets, int32_t *order, int32_t *inv, int32_t *gcnt) {
  return launch_group_full(ctx, ids, T * k, E, counts, offsets, order, inv, nullptr, nullptr, 0,
                           1, nullptr, nullptr, 0, 0, gcnt);
}

// ---------------------------------------------------------------------------
// router_logits_kernel: logits[t][e] = sum_h W[e][h] * x[t][h] for an f32
// router matrix W [E][H] (ffn_gate_inp).  Restates routed_moe's
// self.matvec(ffn_gate_inp) (har-native-qwen35moe.rs:1168-1172), whose F32
// arm is dot_f32_row (:154-163): one f32 accumulator per (token, expert),
// h ascending, each product rounded before it is added (Rust never fuses).
// So every (t, e) is one sequential chain of __fmul_rn/__fadd_rn — bit-exact
// with the reference, which the top-k selection needs.
//
// A CTA covers 32 experts (one per lane) x 32 tokens (4 per thread, 8
// warps), staging 64-wide slices of W (transposed, padded: lane-consecutive
// reads) and of x (warp-broadcast reads) in shared memory; the four tokens'
// chains give each thread four independent adds per W value.
// ---------------------------------------------------------------------------
constexpr int RL_E = 32, RL_WARPS = 8, RL_TPT = 4, RL_TT = RL_WARPS * RL_TPT, RL_KC = 64;

__global__ void __launch_bounds__(RL_WARPS * 32) router_logits_kernel(
    const float *__restrict__ W, const float *__restrict__ x, int64_t T, int E, int H,
    float *__restrict__ logits) {
  __shared__ float ws[RL_KC][RL_E + 1];
  __shared__ __align__(16) float xs[RL_TT][RL_KC];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e0 = blockIdx.x * RL_E;
  const int64_t t0 = (int64_t)blockIdx.y * RL_TT;
  float s[RL_TPT];
#pragma unroll
  for (int j = 0; j < RL_TPT; ++j) s[j] = 0.0f;
  for (int h0 = 0; h0 < H; h0 += RL_KC) {
    const int kc = min(RL_KC, H - h0);
    __syncthreads();  // the previous slice is consumed
    for (int i = threadIdx.x; i < RL_E * RL_KC; i += RL_WARPS * 32) {
      const int r = i / RL_KC, c = i % RL_KC;
      ws[c][r] = (e0 + r < E && c < kc) ? W[(int64_t)(e0 + r) * H + h0 + c] : 0.0f;
      const int64_t t = t0 + r;
      xs[r][c] = (t < T && c < kc) ? x[t * H + h0 + c] : 0.0f;
    }
    __syncthreads();
    const float *xr = xs[warp * RL_TPT];
    for (int c = 0; c < kc; ++c) {
      const float w = ws[c][lane];
#pragma unroll
      for (int j = 0; j < RL_TPT; ++j) s[j] = __fadd_rn(s[j], __fmul_rn(w, xr[j * RL_KC + c]));
    }
  }
  const int e = e0 + lane;
  if (e < E) {
#pragma unroll
    for (int j = 0; j < RL_TPT; ++j) {
      const int64_t t = t0 + warp * RL_TPT + j;
      if (t < T) logits[t * E + e] = s[j];
    }
  }
}

// router_logits_pipe_kernel: the same chains (bit-identical results) for H a
// multiple of 4, with the slices of W and x brought into shared memory by
// cp.async through an RL_S-deep ring, so the L2 latency of slice i+RL_S-1
// overlaps the arithmetic on slice i and the chain runs at its own latency.
// Slices are stored untransposed, [row][h] with a row stride of RL_LD floats:
// lane e reads a float4 of its row (rows 68 floats apart put the eight lanes
// of a quarter-warp on distinct banks), a warp's token rows are broadcast.
constexpr int RL_S = 4, RL_LD = RL_KC + 4;

// NT of a warp's token chains over one staged slice (kc values, a multiple of 4)
template <int NT, int TPT>
__device__ __forceinline__ void rl_slice(const float *wr, const float *xr, int kc,
                                         float (&s)[TPT]) {
#pragma unroll 4
  for (int c = 0; c < kc; c += 4) {
    const float4 w = *reinterpret_cast<const float4 *>(wr + c);
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const float4 v = *reinterpret_cast<const float4 *>(xr + j * RL_LD + c);
      s[j] = __fadd_rn(s[j], __fmul_rn(w.x, v.x));
      s[j] = __fadd_rn(s[j], __fmul_rn(w.y, v.y));
      s[j] = __fadd_rn(s[j], __fmul_rn(w.z, v.z));
      s[j] = __fadd_rn(s[j], __fmul_rn(w.w, v.w));
    }
  }
}
// floats per stage: 32 router rows, then the CTA's 8 * TPT token rows
template <int TPT>
__host__ __device__ constexpr int rl_stage() { return (RL_E + RL_WARPS * TPT) * RL_LD; }

// TPT tokens per thread: 4 for large T (fewer router reads per term), 2 up to
// T = 512 (twice the CTAs, so the SMs hold more warps to hide latency with).
template <int TPT>
__global__ void __launch_bounds__(RL_WARPS * 32) router_logits_pipe_kernel(
    const float *__restrict__ W, const float *__restrict__ x, int64_t T, int E, int H,
    float *__restrict__ logits) {
  constexpr int TT = RL_WARPS * TPT, STAGE = rl_stage<TPT>();
  extern __shared__ __align__(16) float rls[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e0 = blockIdx.x * RL_E;
  const int64_t t0 = (int64_t)blockIdx.y * TT;
  const int nchunk = (H + RL_KC - 1) / RL_KC;
  // issue slice `ch` into ring slot ch % RL_S (16-byte copies; rows past E or
  // T and columns past H are zero-filled and never read by the arithmetic)
  auto load = [&](int ch) {
    float *st = rls + (ch % RL_S) * STAGE;
    const int h0 = ch * RL_KC;
    for (int i = threadIdx.x; i < (RL_E + TT) * (RL_KC / 4); i += RL_WARPS * 32) {
      const int r = i / (RL_KC / 4), c = (i % (RL_KC / 4)) * 4;  // staged row r
      const bool isx = r >= RL_E;
      const bool ok = (isx ? t0 + (r - RL_E) < T : e0 + r < E) && h0 + c < H;
      const float *src = !ok ? W
                         : isx ? x + (t0 + (r - RL_E)) * H + h0 + c
                               : W + (int64_t)(e0 + r) * H + h0 + c;
      tc::cp_async16(st + r * RL_LD + c, src, ok ? 16u : 0u);
    }
  };
#pragma unroll
  for (int ch = 0; ch < RL_S - 1; ++ch) {
    if (ch < nchunk) load(ch);
    tc::cp_async_commit();
  }
  float s[TPT];
#pragma unroll
  for (int j = 0; j < TPT; ++j) s[j] = 0.0f;
  const int64_t left = T - (t0 + warp * TPT);
  const int nt = left <= 0 ? 0 : (left < TPT ? (int)left : TPT);
  for (int ch = 0; ch < nchunk; ++ch) {
    tc::cp_async_wait<RL_S - 2>();  // slice ch has landed (this thread's copies)
    __syncthreads();                // ... everyone's, and slice ch-1 is consumed
    if (ch + RL_S - 1 < nchunk) load(ch + RL_S - 1);
    tc::cp_async_commit();          // (an empty group keeps the count uniform)
    const float *st = rls + (ch % RL_S) * STAGE;
    const float *wr = st + lane * RL_LD, *xr = st + (RL_E + warp * TPT) * RL_LD;
    const int kc = min(RL_KC, H - ch * RL_KC);
    // only the chains of tokens below T: a warp past T only helps load
    if (nt == TPT) {
      rl_slice<TPT>(wr, xr, kc, s);
    } else if (TPT == 4) {
      switch (nt) {
        case 3: rl_slice<3>(wr, xr, kc, s); break;
        case 2: rl_slice<2>(wr, xr, kc, s); break;
        case 1: rl_slice<1>(wr, xr, kc, s); break;
        default: break;
      }
    } else if (nt == 1) {
      rl_slice<1>(wr, xr, kc, s);
    }
  }
  tc::cp_async_wait_all();
  const int e = e0 + lane;
  if (e < E) {
#pragma unroll
    for (int j = 0; j < TPT; ++j) {
      const int64_t t = t0 + warp * TPT + j;
      if (t < T) logits[t * E + e] = s[j];
    }
  }
}

// router_logits_small_kernel: decode-sized batches (T <= RS_T).  The same
// chains again, spread thin: a CTA of RS_W warps owns RS_E experts x RS_T
// tokens, lane (expert e0 + lane/4, token 4*warp + lane%4), so E/RS_E CTAs
// share the router's reads and every chain of a token runs at once.  A chain
// is H dependent adds long, so the kernel is built around keeping that chain
// fed: RS_KC-wide slices of the RS_E router rows and the T token rows come
// through an RS_S-deep cp.async ring, and each thread walks a slice in groups
// of 16 values with the next group's shared-memory loads issued before the
// current group's adds (register double buffering), so no add waits on a load.
//
// For a single token routed_moe's selection is fused in: the CTA that
// finishes last (all logits written and fenced) runs the CTA-wide top-k, then
// re-arms the counter.  Larger decode batches select in route_topk_cta_kernel,
// one CTA per token.
constexpr int RS_E = 8, RS_TW = 4, RS_W = 4, RS_T = RS_TW * RS_W, RS_KC = 128, RS_LD = RS_KC + 4,
              RS_S = 6, RS_G = 16;

// floats of one ring stage (RS_E router rows + the T token rows) and of the
// whole dynamic shared memory (the ring, or E floats per warp for the top-k)
__host__ __device__ inline int rs_stage_floats(int T) { return (RS_E + T) * RS_LD; }
__host__ __device__ inline size_t rs_smem_bytes(int T, int E) {
  const size_t ring = (size_t)RS_S * rs_stage_floats(T), topk = (size_t)E;
  return sizeof(float) * (ring > topk ? ring : topk);
}

__device__ __forceinline__ void rs_group_load(const float *wr, const float *xr, int c, float4 (&w)[RS_G / 4],
                                              float4 (&v)[RS_G / 4]) {
#pragma unroll
  for (int i = 0; i < RS_G / 4; ++i) {
    w[i] = *reinterpret_cast<const float4 *>(wr + c + 4 * i);
    v[i] = *reinterpret_cast<const float4 *>(xr + c + 4 * i);
  }
}
__device__ __forceinline__ float rs_group_chain(float s, const float4 (&w)[RS_G / 4], const float4 (&v)[RS_G / 4]) {
#pragma unroll
  for (int i = 0; i < RS_G / 4; ++i) {
    s = __fadd_rn(s, __fmul_rn(w[i].x, v[i].x));
    s = __fadd_rn(s, __fmul_rn(w[i].y, v[i].y));
    s = __fadd_rn(s, __fmul_rn(w[i].z, v[i].z));
    s = __fadd_rn(s, __fmul_rn(w[i].w, v[i].w));
  }
  return s;
}

__device__ __forceinline__ void rs_load_slice(float *st, const float *W, const float *x, int E, int H,
                                              int e0, int nrows, int h0) {
  for (int i = threadIdx.x; i < nrows * (RS_KC / 4); i += RS_W * 32) {
    const int r = i / (RS_KC / 4), c = 4 * (i % (RS_KC / 4));
    const bool ok = (r < RS_E ? e0 + r < E : true) && h0 + c < H;
    const float *src = !ok ? W : r < RS_E ? W + (int64_t)(e0 + r) * H + h0 + c
                                           : x + (int64_t)(r - RS_E) * H + h0 + c;
    tc::cp_async16(st + r * RS_LD + c, src, ok ? 16u : 0u);
  }
}

__global__ void __launch_bounds__(RS_W * 32, 1) router_logits_small_kernel(
    const float *__restrict__ W, const float *__restrict__ x, int64_t T, int E, int H,
    float *__restrict__ logits, int k, int32_t *__restrict__ ids, float *__restrict__ weights,
    int *counter) {
  extern __shared__ __align__(16) float rss[];
  __shared__ int last_s;
  __shared__ TopkCtaSmem tk_sm;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int el = lane >> 2, tok = RS_TW * warp + (lane & 3);
  const int e0 = blockIdx.x * RS_E;
  const int nt = (int)T, nrows = RS_E + nt, SF = rs_stage_floats(nt);
  const int nchunk = (H + RS_KC - 1) / RS_KC;
  // slice `ch` into ring slot ch % RS_S: nrows rows x RS_KC / 4 16-byte
  // columns over the CTA's threads; rows past E and columns past H are
  // zero-filled and never read by the arithmetic
  auto load = [=](int ch) { rs_load_slice(rss + (ch % RS_S) * SF, W, x, E, H, e0, nrows, ch * RS_KC); };
#pragma unroll
  for (int ch = 0; ch < RS_S - 1; ++ch) {
    if (ch < nchunk) load(ch);
    tc::cp_async_commit();
  }
  const bool active = tok < nt;  // a warp past T only helps load
  float s = 0.0f;
  for (int ch = 0; ch < nchunk; ++ch) {
    tc::cp_async_wait<RS_S - 2>();
    __syncthreads();  // slice ch landed (everyone's copies); slice ch - 1 consumed
    if (ch + RS_S - 1 < nchunk) load(ch + RS_S - 1);
    tc::cp_async_commit();
    if (!active) continue;
    const float *st = rss + (ch % RS_S) * SF;
    const float *wr = st + el * RS_LD, *xr = st + (RS_E + tok) * RS_LD;
    const int kc = min(RS_KC, H - ch * RS_KC);
    if (kc == RS_KC) {
      float4 wa[RS_G / 4], va[RS_G / 4], wb[RS_G / 4], vb[RS_G / 4];
      rs_group_load(wr, xr, 0, wa, va);
#pragma unroll
      for (int g = 0; g < RS_KC / RS_G; g += 2) {
        rs_group_load(wr, xr, (g + 1) * RS_G, wb, vb);
        s = rs_group_chain(s, wa, va);
        if (g + 2 < RS_KC / RS_G) rs_group_load(wr, xr, (g + 2) * RS_G, wa, va);
        s = rs_group_chain(s, wb, vb);
      }
    } else {
      for (int c = 0; c < kc; c += 4) {
        const float4 w = *reinterpret_cast<const float4 *>(wr + c);
        const float4 v = *reinterpret_cast<const float4 *>(xr + c);
        s = __fadd_rn(s, __fmul_rn(w.x, v.x));
        s = __fadd_rn(s, __fmul_rn(w.y, v.y));
        s = __fadd_rn(s, __fmul_rn(w.z, v.z));
        s = __fadd_rn(s, __fmul_rn(w.w, v.w));
      }
    }
  }
  tc::cp_async_wait_all();
  if (active && e0 + el < E) logits[(int64_t)tok * E + e0 + el] = s;
  if (!counter) return;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last_s = atomicAdd(counter, 1) == (int)gridDim.x - 1;
  __syncthreads();
  if (!last_s) return;
  __threadfence();
  // the ring is idle (every copy landed and was read): it holds the exps
  topk_cta_token(logits, E, k, rss, tk_sm, ids, weights);
  __syncthreads();
  if (threadIdx.x == 0) *counter = 0;
}

// router_logits_staged_kernel: the same chains for decode batches whose rows
// fit in shared memory whole ((RS_E + T) rows of H floats).  One warp issues
// every row as RG_CH bulk copies at launch, each H-chunk completing on its own
// mbarrier, so the copies overlap and the computing warps never stop for a
// ring slot or a CTA barrier: each chain waits only for the chunk it reaches.
// Rows are padded by 4 floats so lanes of different rows hit different banks.
// The multiply stays next to its add: on B200 that measured faster (5.7
// cycles per add) than forming a group's products ahead of its adds (6.8);
// the bare chain of adds is 4.4.
constexpr int RG_CH = 8;
constexpr int RG_FULL = 256;  // the chunk of H = 2048
constexpr uint32_t RG_WAIT_LIMIT = 1u << 20;

__host__ __device__ inline int rg_chunk(int H) { return ((H + RG_CH - 1) / RG_CH + 3) & ~3; }
__host__ __device__ inline size_t rg_smem_bytes(int T, int H, int E) {
  const size_t rows = (size_t)(RS_E + T) * (H + 4) * sizeof(float), topk = sizeof(float) * (size_t)E;
  return rows > topk ? rows : topk;
}

__global__ void __launch_bounds__(RS_W * 32, 1) router_logits_staged_kernel(
    const float *__restrict__ W, const float *__restrict__ x, int64_t T, int E, int H,
    float *__restrict__ logits, int k, int32_t *__restrict__ ids, float *__restrict__ weights,
    int *counter, int *status) {
  extern __shared__ __align__(16) float rgs[];
  __shared__ uint64_t full[RG_CH];
  __shared__ int last_s;
  __shared__ TopkCtaSmem tk_sm;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int el = lane >> 2, tok = RS_TW * warp + (lane & 3);
  const int e0 = blockIdx.x * RS_E;
  const int nt = (int)T, LD = H + 4, CH = rg_chunk(H);
  const int ne = min(RS_E, E - e0), nrows = RS_E + nt;
  if (threadIdx.x == 0) {
    for (int c = 0; c < RG_CH; ++c) tc::mbar_init(full + c, 1);
    tc::fence_mbar_init();
  }
  __syncthreads();
  // chunk-major, so the first chunks of every row are in flight first; the
  // router rows (constant) go out before the predecessor has finished, the
  // token rows after it
  auto issue = [&](bool tokens) {
    for (int q = lane; q < RG_CH * nrows; q += 32) {
      const int c = q / nrows, r = q - c * nrows;
      const int h0 = c * CH, n = max(0, min(CH, H - h0));
      if (n == 0 || (r < RS_E && r >= ne) || (r >= RS_E) != tokens) continue;
      const float *src = r < RS_E ? W + (int64_t)(e0 + r) * H + h0 : x + (int64_t)(r - RS_E) * H + h0;
      tc::bulk_g2s(rgs + (size_t)r * LD + h0, src, (uint32_t)(4 * n), full + c);
    }
  };
  if (warp == RS_W - 1) {
    if (lane == 0)
      for (int c = 0; c < RG_CH; ++c) {
        const int h0 = c * CH, n = max(0, min(CH, H - h0));
        tc::mbar_expect_tx(full + c, (uint32_t)(4 * n * (ne + nt)));
      }
    __syncwarp();
    issue(false);
  }
  pdl_wait();
  pdl_launch_dependents();
  if (warp == RS_W - 1) issue(true);
  // A warp with any token runs every lane's chain: lanes past T repeat the
  // last token's (their results are dropped), so the warp runs converged.
  const bool active = tok < nt, run = RS_TW * warp < nt;
  float s = 0.0f;
  bool ok = true;
  if (run) {
    const float *wr = rgs + (size_t)el * LD, *xr = rgs + (size_t)(RS_E + min(tok, nt - 1)) * LD;
    for (int c = 0; c < RG_CH && ok; ++c) {
      const int h0 = c * CH, h1 = min(H, h0 + CH);
      if (h0 >= h1) break;
      // usually landed already: a non-suspending test first
      if (!tc::mbar_test_wait(full + c, 0) && !tc::mbar_wait(full + c, 0, RG_WAIT_LIMIT)) {
        ok = false;
        break;
      }
      auto step = [&](int h) {
        const float4 w = *reinterpret_cast<const float4 *>(wr + h);
        const float4 v = *reinterpret_cast<const float4 *>(xr + h);
        s = __fadd_rn(s, __fmul_rn(w.x, v.x));
        s = __fadd_rn(s, __fmul_rn(w.y, v.y));
        s = __fadd_rn(s, __fmul_rn(w.z, v.z));
        s = __fadd_rn(s, __fmul_rn(w.w, v.w));
      };
      if (h1 - h0 == RG_FULL) {  // the common chunk: a fixed trip count
#pragma unroll 16
        for (int h = 0; h < RG_FULL; h += 4) step(h0 + h);
      } else {
#pragma unroll 4
        for (int h = h0; h < h1; h += 4) step(h);
      }
    }
  }
  // no thread leaves while a copy into this CTA's shared memory may be in flight
  for (int c = 0; c < RG_CH; ++c)
    if (!tc::mbar_wait(full + c, 0, RG_WAIT_LIMIT)) ok = false;
  if (__syncthreads_or(!ok)) {
    if (threadIdx.x == 0) atomicOr(status, DEV_ERR_TIMEOUT);
    return;
  }
  if (active && el < ne) logits[(int64_t)tok * E + e0 + el] = s;
  if (!counter) return;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last_s = atomicAdd(counter, 1) == (int)gridDim.x - 1;
  __syncthreads();
  if (!last_s) return;
  __threadfence();
  topk_cta_token(logits, E, k, rgs, tk_sm, ids, weights);
  __syncthreads();
  if (threadIdx.x == 0) *counter = 0;
}

// Router logits and top-k in one launch for decode batches; *done = false
// (nothing launched) when the shape is not one the fused kernel takes.
int32_t launch_route_fused(har_cuda_ctx *ctx, const float *W, int E, int H, const float *x,
                           int64_t T, int k, float *logits, int32_t *ids, float *weights,
                           bool *done) {
  *done = false;
  const bool vec = H % 4 == 0 && ((uintptr_t)W & 15u) == 0 && ((uintptr_t)x & 15u) == 0;
  if (!vec || T != 1 || E > 8 * TK_T) return HAR_CUDA_OK;
  const size_t gsm = rg_smem_bytes((int)T, H, E);
  if (gsm <= 220 * 1024) {
    cudaFuncSetAttribute(router_logits_staged_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gsm);
    prof_begin(ctx);
    launch_pdl(router_logits_staged_kernel, dim3((unsigned)((E + RS_E - 1) / RS_E)), dim3(RS_W * 32), gsm,
               ctx->stream, W, x, T, E, H, logits, k, ids, weights, ctx->d_status + 1, ctx->d_status);
    *done = true;
    return check_launch(ctx, "router_logits_staged_kernel");
  }
  const size_t smem = rs_smem_bytes((int)T, E);
  if (smem > 227 * 1024) return HAR_CUDA_OK;
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(router_logits_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  prof_begin(ctx);
  router_logits_small_kernel<<<(unsigned)((E + RS_E - 1) / RS_E), RS_W * 32, smem, ctx->stream>>>(
      W, x, T, E, H, logits, k, ids, weights, ctx->d_status + 1);
  *done = true;
  return check_launch(ctx, "router_logits_small_kernel");
}

int32_t launch_router_logits(har_cuda_ctx *ctx, const float *W, int E, int H, const float *x,
                             int64_t T, float *logits) {
  const dim3 grid((unsigned)((E + RL_E - 1) / RL_E), (unsigned)((T + RL_TT - 1) / RL_TT));
  const bool vec = H % 4 == 0 && ((uintptr_t)W & 15u) == 0 && ((uintptr_t)x & 15u) == 0;
  if (vec && T <= RS_T && rg_smem_bytes((int)T, H, E) <= 220 * 1024) {
    const size_t gsm = rg_smem_bytes((int)T, H, E);
    cudaFuncSetAttribute(router_logits_staged_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gsm);
    prof_begin(ctx);
    launch_pdl(router_logits_staged_kernel, dim3((unsigned)((E + RS_E - 1) / RS_E)), dim3(RS_W * 32), gsm,
               ctx->stream, W, x, T, E, H, logits, 0, (int32_t *)nullptr, (float *)nullptr, (int *)nullptr,
               ctx->d_status);
    return check_launch(ctx, "router_logits_staged_kernel");
  }
  if (vec && T <= RS_T) {
    const size_t smem = (size_t)RS_S * rs_stage_floats((int)T) * sizeof(float);
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(router_logits_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    prof_begin(ctx);
    router_logits_small_kernel<<<(unsigned)((E + RS_E - 1) / RS_E), RS_W * 32, smem, ctx->stream>>>(
        W, x, T, E, H, logits, 0, nullptr, nullptr, nullptr);
    return check_launch(ctx, "router_logits_small_kernel");
  }
  if (vec) {
    auto run = [&](auto kern, size_t stage, int tt) {
      const size_t smem = (size_t)RL_S * stage * sizeof(float);
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      const dim3 g((unsigned)((E + RL_E - 1) / RL_E), (unsigned)((T + tt - 1) / tt));
      prof_begin(ctx);
      kern<<<g, RL_WARPS * 32, smem, ctx->stream>>>(W, x, T, E, H, logits);
      return check_launch(ctx, "router_logits_pipe_kernel");
    };
    if (T <= 512) return run(router_logits_pipe_kernel<2>, rl_stage<2>(), RL_WARPS * 2);
    return run(router_logits_pipe_kernel<4>, rl_stage<4>(), RL_WARPS * 4);
  }
  prof_begin(ctx);
  router_logits_kernel<<<grid, RL_WARPS * 32, 0, ctx->stream>>>(W, x, T, E, H, logits);
  return check_launch(ctx, "router_logits_kernel");
}

}  // namespace har
