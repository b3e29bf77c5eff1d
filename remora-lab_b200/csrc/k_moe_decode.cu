// k_moe_decode.cu — the opt-in decode path of the expert FFN
// (HAR_CUDA_MOE_DECODE): compose_moe_route
// (har/crates/har-demo/src/bin/har-native-qwen35moe.rs:979-1048) for a batch
// of at most DECODE_MAX_T tokens in two launches and no grouping pass.
//
// A decode step touches each selected expert for one token, so the expert-major
// grouping, the token gather and the separate combine of the batched path are
// pure overhead there: each is a launch whose fixed cost dwarfs its work.  The
// step is bound by latency, not bandwidth, so every CTA brings ALL its operands
// on chip with a few bulk copies (cp.async.bulk, one round trip) and computes
// from shared memory:
//   1. decode_gate_up_kernel: one CTA per (slot, block of intermediate rows),
//      slot = (token, routed slot) or the token's shared-expert slot; one
//      thread reads the slot's expert id and copies the token's x row and the
//      block's gate and up rows (contiguous in the expert's matrices); the
//      warps compute the rows with the CUDA-core chunk engine
//      (gemv_engine.cuh) and write a = silu(gate . x) * (up . x); the shared
//      slot's first CTA also writes the token's shared gate sigmoid(gate_inp . x);
//   2. decode_down_combine_kernel: one CTA per (token, block of hidden rows);
//      thread j copies slot j's activation row and its expert's down rows of
//      the block; the warps split the (slot, row) dots, and one thread per row
//      adds them as the reference does: routed slots in slot order, each
//      w * value rounded separately, then gate * shared, then the residual.
// f32 activations throughout (HAR's f32 arithmetic, reassociated only inside
// each 64-value chunk as on the CUDA-core GEMV path): the results meet HAR's
// differential verdict.  A token's result does not depend on the other
// tokens of the call.
#include "gemv_engine.cuh"
#include "tc_ptx.cuh"

namespace har {

constexpr int DECODE_MAX_T = 8;
constexpr int DECODE_THREADS = 128;
constexpr int DECODE_MAX_SLOTS = 33;  // k <= 32 routed slots + the shared one
// Rows per CTA.  A decode step's instructions are few and dependent, so the
// kernels need many resident warps per SM to hide latency: small CTAs of
// few rows (gate/up: 4 warps x 8 rows, several CTAs per SM; down: 8 hidden
// rows, two CTAs per SM) rather than large blocks.
constexpr int DECODE_GU_ROWS = 8, DECODE_DOWN_ROWS = 8;
constexpr uint32_t DECODE_WAIT_LIMIT = 1u << 20;  // polls of a copy's barrier
// Activation rows live in shared memory as 64-float chunks in slots of
// DECODE_ACT_LD floats: lane c reads chunk c, and with 272-byte slots the
// eight lanes of a quarter-warp reach eight different bank groups
// (contiguous 256-byte chunks would put all eight on one).  The SwiGLU
// activations are written to scratch in that padded layout, so the down
// kernel copies them as they are; the token rows x are copied whole and
// spread into the padded layout in shared memory (one bulk copy per chunk
// would cost more: the copy engine takes tens of ns per request).
constexpr int DECODE_ACT_LD = 68;
__host__ __device__ inline size_t decode_act_row_bytes(int K) {
  return (size_t)(K / 64) * DECODE_ACT_LD * sizeof(float);
}

struct DecodeArgs {
  const uint8_t *gate, *up, *down, *sh_gate, *sh_up, *sh_down;
  int64_t ebytes_gu, ebytes_d, rb_h, rb_i;
  int E, H, I, T, k, has_shared;
  const float *x, *weights, *gi;  // gi: the shared expert's gate row, or null
  const int32_t *ids;
  float *a;    // [T*k + T][I] SwiGLU activations (routed slots, then shared)
  float *gsh;  // [T] shared gate
  float *y;
  int add_residual;
  int *status;
};

template <int LPR, int CPL>
__global__ void __launch_bounds__(DECODE_THREADS, CPL == 1 ? 5 : 2) decode_gate_up_kernel(DecodeArgs p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t bar;
  __shared__ int skip;
  constexpr int RPW = 32 / LPR, R = DECODE_GU_ROWS, NW = DECODE_THREADS / 32;
  constexpr int QN = R / (NW * RPW) > 0 ? R / (NW * RPW) : 1;  // row passes per warp
  const int nb = (p.I + R - 1) / R;
  const int slot = blockIdx.x / nb, blk = blockIdx.x - slot * nb;
  const int n = p.T * p.k;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = blk * R, nr = min(p.I - r0, R);
  const int t = slot < n ? slot / p.k : slot - n;
  const float *xt = p.x + (int64_t)t * p.H;
  float *xraw = reinterpret_cast<float *>(smem);
  float *xs = xraw + p.H;
  uint8_t *wg_s = smem + ((4 * (size_t)p.H + decode_act_row_bytes(p.H) + 127) & ~(size_t)127);
  uint8_t *wu_s = wg_s + (size_t)R * p.rb_h;
  const uint32_t wb = (uint32_t)(nr * p.rb_h), xb = (uint32_t)(4 * p.H);
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    tc::fence_mbar_init();
    if (slot >= n) {  // the shared expert's rows: constant, wanted before the predecessor ends
      tc::mbar_expect_tx(&bar, xb + 2 * wb);
      tc::bulk_g2s(wg_s, p.sh_gate + (int64_t)r0 * p.rb_h, wb, &bar);
      tc::bulk_g2s(wu_s, p.sh_up + (int64_t)r0 * p.rb_h, wb, &bar);
    }
  }
  pdl_wait();  // ids and x come from earlier launches
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    int bad = 0;
    if (slot < n) {
      const int e = p.ids[slot];
      bad = e < 0 || e >= p.E;
      if (bad && blk == 0) atomicOr(p.status, DEV_ERR_BOUNDS);
      if (!bad) {
        tc::mbar_expect_tx(&bar, xb + 2 * wb);
        tc::bulk_g2s(wg_s, p.gate + (int64_t)e * p.ebytes_gu + (int64_t)r0 * p.rb_h, wb, &bar);
        tc::bulk_g2s(wu_s, p.up + (int64_t)e * p.ebytes_gu + (int64_t)r0 * p.rb_h, wb, &bar);
      }
    }
    skip = bad;
    if (!bad) tc::bulk_g2s(xraw, xt, xb, &bar);
  }
  __syncthreads();
  if (skip) return;  // an out-of-range expert id: the slot contributes nothing
  if (slot >= n && blk == 0 && warp == 0 && p.gi) {  // overlaps the copies
    const float g = shared_gate_warp(p.gi, xt, p.H, lane);
    if (lane == 0) p.gsh[t] = g;
  }
  const bool landed = tc::mbar_wait(&bar, 0, DECODE_WAIT_LIMIT);
  if (!landed && threadIdx.x == 0) atomicOr(p.status, DEV_ERR_TIMEOUT);
  if (__syncthreads_or(!landed)) return;
  for (int q = threadIdx.x; q < p.H / 4; q += DECODE_THREADS)  // x into the padded layout
    reinterpret_cast<float4 *>(xs + DECODE_ACT_LD * (q >> 4))[q & 15] = reinterpret_cast<const float4 *>(xraw)[q];
  __syncthreads();
  const int grp = lane / LPR, gl = lane % LPR;
  const int C = p.H / 64;
  LaneAct<ACT_F32> act[CPL];
#pragma unroll
  for (int i = 0; i < CPL; ++i)
    if (gl + LPR * i < C) act[i].load_row(xs + DECODE_ACT_LD * (gl + LPR * i));
  // This warp's QN row passes of gate then up, one dot per iteration.  The
  // loop stays rolled on purpose: each launch runs once per layer on SMs whose
  // instruction caches hold other kernels, so one static copy of the chunk
  // dot fetched once beats unrolled copies that are each fetched from L2.
  float *arow = p.a + (int64_t)slot * ((p.I / 64) * DECODE_ACT_LD);
  float g = 0.0f;
#pragma unroll 1
  for (int it = 0; it < 2 * QN; ++it) {
    const int q = it >> 1, r = (q * NW + warp) * RPW + grp;
    const uint8_t *row = ((it & 1) ? wu_s : wg_s) + (int64_t)(r < nr ? r : 0) * p.rb_h;
    float v = 0.0f;
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      const int ch = gl + LPR * i;
      if (ch < C) v += chunk_dot_ilp(load_wchunk_s(row, ch), ch, act[i]);
    }
    v = lane_group_sum<LPR>(v);
    if (!(it & 1)) {
      g = v;
    } else if (r < nr && gl == 0) {
      const int ri = r0 + r;  // padded position of intermediate row ri
      arow[DECODE_ACT_LD * (ri >> 6) + (ri & 63)] = __fmul_rn(g / (1.0f + expf(-g)), v);
    }
  }
}

// The down kernel runs one warp per slot, up to decode_down_warps(CPL) warps
// (more slots wrap around), two CTAs per SM; two chunks per lane need the
// registers of a smaller CTA.
__host__ __device__ constexpr int decode_down_warps(int cpl) { return cpl == 1 ? 12 : 8; }

template <int LPR, int CPL>
__global__ void __launch_bounds__(decode_down_warps(CPL) * 32, CPL == 1 ? 2 : 1) decode_down_combine_kernel(DecodeArgs p,
                                                                                          int rows_per_cta) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int RPW = 32 / LPR, QD = DECODE_DOWN_ROWS / RPW > 0 ? DECODE_DOWN_ROWS / RPW : 1;
  __shared__ uint64_t bar;
  __shared__ uint8_t ok_s[DECODE_MAX_SLOTS];
  __shared__ float swt[DECODE_MAX_SLOTS];
  __shared__ float part[DECODE_MAX_SLOTS][DECODE_DOWN_ROWS];
  const int R = rows_per_cta;
  const int nb = (p.H + R - 1) / R;
  const int t = blockIdx.x / nb, blk = blockIdx.x - t * nb;
  const int n = p.T * p.k, ns = p.k + p.has_shared;
  const int nw = (int)(blockDim.x >> 5), warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = blk * R, nr = min(p.H - r0, R);
  float *as = reinterpret_cast<float *>(smem);
  const int SLD = (p.I / 64) * DECODE_ACT_LD;  // floats per staged activation row
  uint8_t *w_s = smem + (((size_t)ns * decode_act_row_bytes(p.I) + 127) & ~(size_t)127);
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, ns);
    tc::fence_mbar_init();
  }
  __syncthreads();
  const uint32_t rb = (uint32_t)(4 * SLD);
  if (threadIdx.x < ns) {
    // slot j's expert: its down rows r0 .. r0 + nr - 1.  The ids and weights
    // come from two or more launches back, so these copies start before the
    // gate/up launch has finished.
    const int j = threadIdx.x;
    const uint8_t *wd = p.sh_down;
    bool ok = true;
    if (j < p.k) {
      const int s = t * p.k + j, e = p.ids[s];
      ok = e >= 0 && e < p.E;  // a bad id contributes nothing (gate/up reported it)
      wd = p.down + (int64_t)(ok ? e : 0) * p.ebytes_d;
      swt[j] = p.weights[s];
    }
    ok_s[j] = ok;
    const uint32_t wb = ok ? (uint32_t)(nr * p.rb_i) : 0u;
    tc::mbar_expect_tx(&bar, wb + (j == 0 ? (uint32_t)ns * rb : 0u));
    if (ok) tc::bulk_g2s(w_s + (size_t)j * R * p.rb_i, wd + (int64_t)r0 * p.rb_i, wb, &bar);
  }
  pdl_wait();  // the activations and the shared gate are the gate/up launch's
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    // the token's activation rows (its k routed slots are contiguous)
    tc::bulk_g2s(as, p.a + (int64_t)t * p.k * SLD, (uint32_t)p.k * rb, &bar);
    if (p.has_shared) {
      tc::bulk_g2s(as + (size_t)p.k * SLD, p.a + (int64_t)(n + t) * SLD, rb, &bar);
      swt[p.k] = p.gi ? p.gsh[t] : 1.0f;
    }
  }
  const bool landed = tc::mbar_wait(&bar, 0, DECODE_WAIT_LIMIT);
  if (!landed && threadIdx.x == 0) atomicOr(p.status, DEV_ERR_TIMEOUT);
  if (__syncthreads_or(!landed)) return;  // (also publishes ok_s / swt)
  const int grp = lane / LPR, gl = lane % LPR;
  const int C = p.I / 64;
  for (int j = warp; j < ns; j += nw) {
    if (!ok_s[j]) continue;
    LaneAct<ACT_F32> act[CPL];
#pragma unroll
    for (int i = 0; i < CPL; ++i)
      if (gl + LPR * i < C) act[i].load_row(as + (size_t)j * SLD + DECODE_ACT_LD * (gl + LPR * i));
#pragma unroll 1
    for (int q = 0; q < QD; ++q) {  // rolled, as in the gate/up kernel
      const int r = q * RPW + grp;
      const uint8_t *row = w_s + ((size_t)j * R + (r < nr ? r : 0)) * p.rb_i;
      float v = 0.0f;
#pragma unroll
      for (int i = 0; i < CPL; ++i) {
        const int ch = gl + LPR * i;
        if (ch < C) v += chunk_dot_ilp(load_wchunk_s(row, ch), ch, act[i]);
      }
      v = lane_group_sum<LPR>(v);
      if (gl == 0 && r < nr) part[j][r] = v;
    }
  }
  __syncthreads();
  if (threadIdx.x < nr) {
    const int r = threadIdx.x;
    float routed = 0.0f;
    for (int j = 0; j < p.k; ++j)
      if (ok_s[j]) routed = __fadd_rn(routed, __fmul_rn(swt[j], part[j][r]));  // output += weight * value
    float out = p.has_shared ? __fadd_rn(routed, __fmul_rn(swt[p.k], part[p.k][r])) : routed;
    if (p.add_residual) out = __fadd_rn(p.x[(int64_t)t * p.H + r0 + r], out);
    p.y[(int64_t)t * p.H + r0 + r] = out;
  }
}

template <template <int, int> class KF, typename Launch>
static int32_t dispatch_shape(har_cuda_ctx *ctx, int K, Launch &&launch) {
  const GemvShape s = gemv_shape(K);
  if (s.LPR == 4) return launch(KF<4, 1>::get());
  if (s.LPR == 8) return launch(KF<8, 1>::get());
  if (s.LPR == 16) return launch(KF<16, 1>::get());
  if (s.CPL == 1) return launch(KF<32, 1>::get());
  if (s.CPL == 2) return launch(KF<32, 2>::get());
  return set_error(ctx, HAR_CUDA_ERR_UNSUPPORTED, "moe decode: row length above 4096");
}

template <int LPR, int CPL>
struct GateUpK {
  static decltype(&decode_gate_up_kernel<LPR, CPL>) get() { return &decode_gate_up_kernel<LPR, CPL>; }
};
template <int LPR, int CPL>
struct DownK {
  static decltype(&decode_down_combine_kernel<LPR, CPL>) get() {
    return &decode_down_combine_kernel<LPR, CPL>;
  }
};

size_t moe_decode_scratch_bytes(const har_cuda_moe_layer *layer, int64_t T, int k) {
  const size_t a = (size_t)(T * k + T) * decode_act_row_bytes((int)layer->I);
  return ((a + 255) & ~(size_t)255) + 4 * (size_t)T + 256;
}

int32_t run_moe_decode(har_cuda_ctx *ctx, const har_cuda_moe_layer *layer, const float *x,
                       int64_t T, int k, const int32_t *ids, const float *weights, float *y,
                       uint32_t flags, uint8_t *S) {
  if (T > DECODE_MAX_T)
    return set_error(ctx, HAR_CUDA_ERR_GEOMETRY,
                     "moe_ffn: HAR_CUDA_MOE_DECODE serves at most " + std::to_string(DECODE_MAX_T) +
                         " tokens per call");
  if (k > 32) return set_error(ctx, HAR_CUDA_ERR_GEOMETRY, "moe_ffn: HAR_CUDA_MOE_DECODE needs k <= 32");
  if (((uintptr_t)x & 15u) || ((uintptr_t)y & 15u))
    return set_error(ctx, HAR_CUDA_ERR_ARG, "moe_ffn: x and y must be 16-byte aligned");
  // the kernels copy row blocks with cp.async.bulk: 16-byte aligned sources
  for (const har_cuda_weights *w : {layer->gate, layer->up, layer->down, layer->sh_gate,
                                    layer->sh_up, layer->sh_down})
    if (w && ((uintptr_t)w->dev & 15u))
      return set_error(ctx, HAR_CUDA_ERR_ARG,
                       "moe_ffn: HAR_CUDA_MOE_DECODE needs 16-byte aligned weight buffers");
  DecodeArgs p{};
  p.gate = layer->gate->dev;
  p.up = layer->up->dev;
  p.down = layer->down->dev;
  p.has_shared = layer->sh_gate ? 1 : 0;
  p.sh_gate = p.has_shared ? layer->sh_gate->dev : nullptr;
  p.sh_up = p.has_shared ? layer->sh_up->dev : nullptr;
  p.sh_down = p.has_shared ? layer->sh_down->dev : nullptr;
  p.ebytes_gu = layer->gate->expert_bytes;
  p.ebytes_d = layer->down->expert_bytes;
  p.rb_h = layer->gate->row_bytes;
  p.rb_i = layer->down->row_bytes;
  p.E = (int)layer->E;
  p.H = (int)layer->H;
  p.I = (int)layer->I;
  p.T = (int)T;
  p.k = k;
  p.x = x;
  p.weights = weights;
  p.ids = ids;
  p.gi = p.has_shared ? layer->sh_gate_inp : nullptr;
  const size_t a_bytes = ((size_t)(T * k + T) * decode_act_row_bytes(p.I) + 255) & ~(size_t)255;
  p.a = reinterpret_cast<float *>(S);
  p.gsh = reinterpret_cast<float *>(S + a_bytes);
  p.y = y;
  p.add_residual = (flags & HAR_CUDA_MOE_ADD_RESIDUAL) ? 1 : 0;
  p.status = ctx->d_status;
  const int slots = (int)(T * k) + (p.has_shared ? (int)T : 0);
  const int ns = k + p.has_shared;
  constexpr size_t SMEM_MAX = 227 * 1024;
  const size_t smem_gu = ((4 * (size_t)p.H + decode_act_row_bytes(p.H) + 127) & ~(size_t)127) +
                        2 * (size_t)DECODE_GU_ROWS * p.rb_h;
  if (smem_gu > SMEM_MAX)
    return set_error(ctx, HAR_CUDA_ERR_UNSUPPORTED, "moe_ffn: HAR_CUDA_MOE_DECODE: hidden size too large");
  // down rows per CTA: DECODE_DOWN_ROWS, halved until the slots' rows fit
  int rpc_d = DECODE_DOWN_ROWS;
  auto smem_d = [&](int r) {
    return (((size_t)ns * decode_act_row_bytes(p.I) + 127) & ~(size_t)127) + (size_t)ns * r * p.rb_i;
  };
  while (rpc_d > 1 && smem_d(rpc_d) > SMEM_MAX) rpc_d /= 2;
  if (smem_d(rpc_d) > SMEM_MAX)
    return set_error(ctx, HAR_CUDA_ERR_GEOMETRY, "moe_ffn: HAR_CUDA_MOE_DECODE: (k + 1) x I too large");
  int32_t st = dispatch_shape<GateUpK>(ctx, p.H, [&](auto kern) -> int32_t {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_gu);
    prof_begin(ctx);
    launch_pdl(kern, dim3((unsigned)(slots * ((p.I + DECODE_GU_ROWS - 1) / DECODE_GU_ROWS))),
               dim3(DECODE_THREADS), smem_gu, ctx->stream, p);
    return check_launch(ctx, "decode_gate_up_kernel");
  });
  if (st) return st;
  return dispatch_shape<DownK>(ctx, p.I, [&](auto kern) -> int32_t {
    const size_t smem = smem_d(rpc_d);
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    prof_begin(ctx);
    const int wmax = decode_down_warps(gemv_shape(p.I).CPL), warps = ns < wmax ? ns : wmax;
    launch_pdl(kern, dim3((unsigned)(T * ((p.H + rpc_d - 1) / rpc_d))), dim3(32 * warps), smem, ctx->stream, p,
               rpc_d);
    return check_launch(ctx, "decode_down_combine_kernel");
  });
}

}  // namespace har
