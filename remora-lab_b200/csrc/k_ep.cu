// k_ep.cu — expert parallelism: the MoE FFN layer with its routed experts
// sharded over the G ranks of one box, token rows dispatched to the experts'
// ranks and partial results combined back with NCCL over NVLink.
//
// The reference runs every expert of a layer on one CPU
// (compose_moe_route, har/crates/har-demo/src/bin/har-native-qwen35moe.rs:979-1048);
// this is the router-to-expert dispatch of a sharded deployment, so it has no
// reference counterpart: per layer and rank r (E/G routed experts each, expert
// e on rank e / (E/G); the shared expert replicated on every rank):
//   1. ep_plan_kernel: for every destination d and local token t, the row
//      (d, t) carries x[t] and t's k slots as d-local expert ids (-1 where the
//      expert lives elsewhere) with their routing weights.  Every rank sends
//      exactly T rows to every rank (rows without a local expert carry stale
//      data and are skipped, except the rows a rank sends itself, which its
//      shared expert reads), so no count exchange or host sync is needed and
//      the whole layer can be captured in a CUDA graph;
//   2. one grouped NCCL send/recv round moves the rows (x, ids, weights);
//   3. the expert pipeline runs on the G*T received rows with the rank's shard
//      (empty slots allowed, no residual): each row's output is the partial
//      sum over its slots that live here.  The shared expert is the
//      pipeline's shared expert for the rank's own T rows among them (rows
//      rank*T ..), weighted by sigmoid(gate_inp . x): its token tiles join the
//      routed experts' tensor-core launches;
//   4. a second round returns the partial sums to the tokens' ranks;
//   5. ep_combine_kernel adds the residual and the G partial sums in rank
//      order (the rank's own partial holds the shared expert).
// Results match the single-GPU layer up to f32 summation order (the routed
// terms are summed per rank, then across ranks).
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <thread>
#include <climits>
#include <cstring>
#include <string>

#include "har_internal.cuh"

struct har_cuda_ep {
  int world = 1, rank = 0, device = 0;
  ncclComm_t comm = nullptr;  // non-blocking: every NCCL call is polled against a deadline
  int64_t op_timeout_ms = 60000;  // bound on an exchange's host-side enqueue
  void *buf = nullptr;  // exchange buffers, grown on demand
  size_t bytes = 0;
  // the exchanges run on their own stream, joined to the caller's by events,
  // so the shared expert computes while the dispatch moves rows
  cudaStream_t cs = nullptr;
  cudaEvent_t ev[4] = {nullptr, nullptr, nullptr, nullptr};  // plan, dispatch, local, return
};

namespace har {

static int32_t nccl_error(har_cuda_ctx *ctx, const char *what, ncclResult_t r) {
  return set_error(ctx, HAR_CUDA_ERR_NCCL, std::string(what) + ": " + ncclGetErrorString(r));
}

// The communicator is non-blocking (ncclConfig_t::blocking = 0): an NCCL call
// may return ncclInProgress and finish in the background.  Poll its state
// until it settles or `timeout_ms` passes; on expiry abort the communicator
// (every rank's later calls then fail instead of waiting for a peer that will
// never come) and report HAR_CUDA_ERR_TIMEOUT.  The same bound covers a
// communicator's creation, which waits for every rank to join.
static int32_t nccl_settle(har_cuda_ctx *ctx, ncclComm_t *comm, ncclResult_t r, const char *what,
                           int64_t timeout_ms) {
  if (r != ncclSuccess && r != ncclInProgress) return nccl_error(ctx, what, r);
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    ncclResult_t state = ncclSuccess;
    const ncclResult_t q = ncclCommGetAsyncError(*comm, &state);
    if (q != ncclSuccess) return nccl_error(ctx, "ncclCommGetAsyncError", q);
    if (state == ncclSuccess) return HAR_CUDA_OK;
    if (state != ncclInProgress) return nccl_error(ctx, what, state);
    const int64_t ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                           std::chrono::steady_clock::now() - t0).count();
    if (ms > timeout_ms) {
      ncclCommAbort(*comm);
      *comm = nullptr;
      return set_error(ctx, HAR_CUDA_ERR_TIMEOUT,
                       std::string(what) + " did not complete within " + std::to_string(timeout_ms) +
                           " ms (a rank missing or gone); the communicator was aborted");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(100));
  }
}

// Row (d, t) of the dispatch: d-local ids and weights of token t's slots, and
// x[t] when at least one slot lives on d.
__global__ void __launch_bounds__(128) ep_plan_kernel(const float *__restrict__ x, int H,
                                                      const int32_t *__restrict__ ids,
                                                      const float *__restrict__ w, int T, int k,
                                                      int E, int El, float *__restrict__ sx,
                                                      int32_t *__restrict__ sids,
                                                      float *__restrict__ sw, int keep, int *status) {
  const int d = blockIdx.x / T, t = blockIdx.x % T;
  const int64_t row = (int64_t)d * T + t;
  __shared__ int any;
  if (threadIdx.x == 0) any = 0;
  __syncthreads();
  for (int j = threadIdx.x; j < k; j += blockDim.x) {
    const int e = ids[(int64_t)t * k + j];
    int loc = -1;
    if (e < 0 || e >= E) {
      atomicOr(status, DEV_ERR_BOUNDS);
    } else if (e / El == d) {
      loc = e - d * El;
      any = 1;
    }
    sids[row * k + j] = loc;
    sw[row * k + j] = loc >= 0 ? w[(int64_t)t * k + j] : 0.0f;
  }
  __syncthreads();
  if (!any && d != keep) return;  // rows to `keep` always carry x (its shared expert reads them)
  const float4 *src = reinterpret_cast<const float4 *>(x + (int64_t)t * H);
  float4 *dst = reinterpret_cast<float4 *>(sx + row * H);
  for (int i = threadIdx.x; i < H / 4; i += blockDim.x) dst[i] = src[i];
}

// y[t] = (x[t] with the residual flag) + shared[t] (when given) + sum_d back[d][t].
__global__ void __launch_bounds__(256) ep_combine_kernel(const float *x, int H, int T, int G,
                                                         const float *__restrict__ ysh,
                                                         const float *__restrict__ back,
                                                         int residual, float *y) {
  const int t = blockIdx.x;
  for (int h = threadIdx.x; h < H; h += blockDim.x) {
    const int64_t i = (int64_t)t * H + h;
    float acc = residual ? x[i] : 0.0f;
    if (ysh) acc = __fadd_rn(acc, ysh[i]);
    for (int d = 0; d < G; ++d) acc = __fadd_rn(acc, back[((int64_t)d * T + t) * H + h]);
    y[i] = acc;
  }
}

}  // namespace har

using namespace har;

namespace {

size_t al256(size_t v) { return (v + 255) & ~(size_t)255; }

struct EpLayout {
  size_t sx, sids, sw, rx, rids, rw, part, back, total;
};

EpLayout ep_layout(int G, int64_t T, int k, int64_t H) {
  EpLayout L;
  size_t off = 0;
  auto take = [&](size_t b) { size_t o = off; off += al256(b); return o; };
  const size_t rows = (size_t)G * (size_t)T;
  L.sx = take(4 * rows * H);
  L.sids = take(4 * rows * k);
  L.sw = take(4 * rows * k);
  L.rx = take(4 * rows * H);
  L.rids = take(4 * rows * k);
  L.rw = take(4 * rows * k);
  L.part = take(4 * rows * H);
  L.back = take(4 * rows * H);
  L.total = off;
  return L;
}

int32_t ep_reserve(har_cuda_ctx *ctx, har_cuda_ep *ep, size_t bytes) {
  if (ep->bytes >= bytes) return HAR_CUDA_OK;
  if (ep->buf) {
    cudaStreamSynchronize(ctx->stream);
    cudaFree(ep->buf);
    ep->buf = nullptr;
    ep->bytes = 0;
  }
  if (cudaMalloc(&ep->buf, bytes) != cudaSuccess)
    return set_error(ctx, HAR_CUDA_ERR_OOM, "ep: exchange buffer allocation failed");
  ep->bytes = bytes;
  return HAR_CUDA_OK;
}

// One all-to-all round: `n` elements of `type` from send + d*n to rank d,
// received into recv + d*n from rank d, for every d.
int32_t ep_all_to_all(har_cuda_ctx *ctx, har_cuda_ep *ep, const void *send, void *recv, size_t n,
                      ncclDataType_t type, size_t esize) {
  for (int d = 0; d < ep->world; ++d) {
    ncclResult_t r = ncclSend((const uint8_t *)send + (size_t)d * n * esize, n, type, d, ep->comm,
                              ep->cs);
    if (r != ncclSuccess && r != ncclInProgress) return nccl_error(ctx, "ncclSend", r);
    r = ncclRecv((uint8_t *)recv + (size_t)d * n * esize, n, type, d, ep->comm, ep->cs);
    if (r != ncclSuccess && r != ncclInProgress) return nccl_error(ctx, "ncclRecv", r);
  }
  return HAR_CUDA_OK;
}

int32_t ep_layer(har_cuda_ctx *ctx, har_cuda_ep *ep, const har_cuda_moe_layer *local,
                 const har_cuda_moe_layer *shared, const float *gate_inp, const float *x,
                 int64_t T, int k, const int32_t *ids, const float *w, float *y, uint32_t flags) {
  const int G = ep->world;
  const int64_t H = local->H;
  const int El = (int)local->E, E = El * G;
  const EpLayout L = ep_layout(G, T, k, H);
  int32_t st = ep_reserve(ctx, ep, L.total);
  if (st) return st;
  const uint32_t mode0 = flags & (HAR_CUDA_MOE_ACT_Q8K | HAR_CUDA_MOE_FORCE_GEMV |
                                  HAR_CUDA_MOE_FORCE_TC | HAR_CUDA_MOE_TC_F16W);
  // The shared expert joins the rank's routed experts as the layer's shared
  // expert, serving only the rank's own rows among the received ones (rows
  // rank*T .. rank*T + T - 1: every rank sends its T rows to every rank, this
  // one included), so one expert pipeline covers both: its token tiles share
  // the tensor-core launches with the routed tiles.
  har_cuda_moe_layer comb;
  const har_cuda_moe_layer *lay = local;
  if (shared) {
    comb.gate = local->gate;
    comb.up = local->up;
    comb.down = local->down;
    comb.sh_gate = shared->gate;
    comb.sh_up = shared->up;
    comb.sh_down = shared->down;
    comb.sh_gate_inp = gate_inp;
    comb.E = local->E;
    comb.H = local->H;
    comb.I = local->I;
    comb.tc_maps = local->tc_maps && shared->tc_maps;
    comb.map_gate = local->map_gate;
    comb.map_up = local->map_up;
    comb.map_down = local->map_down;
    comb.map_sh_gate = shared->map_gate;
    comb.map_sh_up = shared->map_up;
    comb.map_sh_down = shared->map_down;
    lay = &comb;
  }
  const uint32_t lmode = mode0 | HAR_CUDA_MOE_EMPTY_SLOTS;
  if ((st = ensure_scratch(ctx, moe_scratch_bytes(ctx, lay, (int64_t)G * T, k, lmode)))) return st;
  uint8_t *B = (uint8_t *)ep->buf;
  float *sx = (float *)(B + L.sx), *sw = (float *)(B + L.sw), *rx = (float *)(B + L.rx);
  float *rw = (float *)(B + L.rw), *part = (float *)(B + L.part), *back = (float *)(B + L.back);
  int32_t *sids = (int32_t *)(B + L.sids), *rids = (int32_t *)(B + L.rids);
  // Compute runs on ctx->stream, the exchanges on ep->cs; events order them:
  // plan -> dispatch -> experts -> return -> combine.  The same order holds
  // under CUDA-graph capture (fork and join).
  auto join = [&](cudaStream_t from, cudaStream_t to, cudaEvent_t e) -> int32_t {
    if (cudaEventRecord(e, from) != cudaSuccess || cudaStreamWaitEvent(to, e, 0) != cudaSuccess)
      return set_error(ctx, HAR_CUDA_ERR_CUDA, "ep: stream ordering failed");
    return HAR_CUDA_OK;
  };
  // 1. plan
  prof_begin(ctx);
  ep_plan_kernel<<<(unsigned)(G * T), 128, 0, ctx->stream>>>(x, (int)H, ids, w, (int)T, k, E, El,
                                                            sx, sids, sw, shared ? ep->rank : -1,
                                                            ctx->d_status);
  if ((st = check_launch(ctx, "ep_plan_kernel"))) return st;
  if ((st = join(ctx->stream, ep->cs, ep->ev[0]))) return st;
  // 2. dispatch (exchange stream)
  ncclResult_t r = ncclGroupStart();
  if (r != ncclSuccess) return nccl_error(ctx, "ncclGroupStart", r);
  st = ep_all_to_all(ctx, ep, sx, rx, (size_t)T * H, ncclFloat32, 4);
  if (!st) st = ep_all_to_all(ctx, ep, sids, rids, (size_t)T * k, ncclInt32, 4);
  if (!st) st = ep_all_to_all(ctx, ep, sw, rw, (size_t)T * k, ncclFloat32, 4);
  r = ncclGroupEnd();
  if (st) return st;
  if ((st = nccl_settle(ctx, &ep->comm, r, "ep dispatch", ep->op_timeout_ms))) return st;
  // 3. the rank's experts on the received rows (partial sums per row), with
  // the shared expert on the rank's own rows
  if ((st = join(ep->cs, ctx->stream, ep->ev[1]))) return st;
  if ((st = run_moe_ffn_range(ctx, lay, rx, (int64_t)G * T, k, rids, rw, part, lmode,
                              (uint8_t *)ctx->scratch, shared ? (int64_t)ep->rank * T : 0,
                              shared ? T : 0)))
    return st;
  if ((st = join(ctx->stream, ep->cs, ep->ev[2]))) return st;
  // 4. return the partial sums (exchange stream)
  r = ncclGroupStart();
  if (r != ncclSuccess) return nccl_error(ctx, "ncclGroupStart", r);
  st = ep_all_to_all(ctx, ep, part, back, (size_t)T * H, ncclFloat32, 4);
  r = ncclGroupEnd();
  if (st) return st;
  if ((st = nccl_settle(ctx, &ep->comm, r, "ep return", ep->op_timeout_ms))) return st;
  if ((st = join(ep->cs, ctx->stream, ep->ev[3]))) return st;
  // 5. residual + partials in rank order (this rank's holds the shared expert)
  prof_begin(ctx);
  ep_combine_kernel<<<(unsigned)T, 256, 0, ctx->stream>>>(
      x, (int)H, (int)T, G, nullptr, back, (flags & HAR_CUDA_MOE_ADD_RESIDUAL) ? 1 : 0, y);
  return check_launch(ctx, "ep_combine_kernel");
}

int32_t ep_check(har_cuda_ctx *ctx, har_cuda_ep *ep, const har_cuda_moe_layer *local,
                 const har_cuda_moe_layer *shared, int64_t T, int k, uint32_t flags) {
  if (!ctx) return HAR_CUDA_ERR_ARG;
  if (!ep || !ep->comm)
    return set_error(ctx, HAR_CUDA_ERR_NOT_INIT, "ep: no communicator (never created, or aborted)");
  if (ep->device != ctx->device)
    return set_error(ctx, HAR_CUDA_ERR_ARG, "ep: communicator belongs to another device");
  if (!local) return set_error(ctx, HAR_CUDA_ERR_ARG, "ep: local layer is null");
  if (local->sh_gate)
    return set_error(ctx, HAR_CUDA_ERR_ARG,
                     "ep: the local layer holds routed experts only (pass the shared expert "
                     "as the one-expert shared layer)");
  if (shared && (shared->E != 1 || shared->H != local->H || shared->sh_gate))
    return set_error(ctx, HAR_CUDA_ERR_GEOMETRY, "ep: the shared layer must be one expert of H");
  if (T < 0 || k <= 0 || k > local->E * (int64_t)ep->world)
    return set_error(ctx, HAR_CUDA_ERR_GEOMETRY, "ep: need T >= 0 and 0 < k <= E");
  if ((int64_t)ep->world * T * k > ((int64_t)1 << 24))
    return set_error(ctx, HAR_CUDA_ERR_GEOMETRY, "ep: G*T*k <= 2^24");
  if (local->H % 4)
    return set_error(ctx, HAR_CUDA_ERR_GEOMETRY, "ep: hidden size must be a multiple of 4");
  if ((flags & HAR_CUDA_MOE_FORCE_GEMV) && (flags & HAR_CUDA_MOE_FORCE_TC))
    return set_error(ctx, HAR_CUDA_ERR_ARG, "ep: FORCE_GEMV and FORCE_TC are exclusive");
  if ((flags & HAR_CUDA_MOE_ACT_Q8K) && (flags & HAR_CUDA_MOE_FORCE_TC))
    return set_error(ctx, HAR_CUDA_ERR_UNSUPPORTED,
                     "ep: the tensor-core path has no Q8_K activation mode");
  if (flags & ~(HAR_CUDA_MOE_ADD_RESIDUAL | HAR_CUDA_MOE_ACT_Q8K | HAR_CUDA_MOE_FORCE_GEMV |
                HAR_CUDA_MOE_FORCE_TC | HAR_CUDA_MOE_TC_F16W))
    return set_error(ctx, HAR_CUDA_ERR_ARG, "ep: unknown flag bits");
  return HAR_CUDA_OK;
}

}  // namespace

extern "C" {

int32_t har_cuda_ep_unique_id(uint8_t *out, size_t len) {
  if (!out || len < sizeof(ncclUniqueId)) return HAR_CUDA_ERR_ARG;
  ncclUniqueId id;
  if (ncclGetUniqueId(&id) != ncclSuccess) return HAR_CUDA_ERR_NCCL;
  memcpy(out, &id, sizeof(id));
  return HAR_CUDA_OK;
}

int32_t har_cuda_ep_create_timeout(har_cuda_ctx *ctx, const uint8_t *unique_id, size_t len,
                                   int32_t world, int32_t rank, int64_t timeout_ms,
                                   har_cuda_ep **out) {
  if (!ctx || !unique_id || !out || len < sizeof(ncclUniqueId)) return HAR_CUDA_ERR_ARG;
  *out = nullptr;
  if (world < 1 || rank < 0 || rank >= world)
    return set_error(ctx, HAR_CUDA_ERR_ARG, "ep_create: need 0 <= rank < world");
  if (timeout_ms <= 0) return set_error(ctx, HAR_CUDA_ERR_ARG, "ep_create: timeout_ms must be positive");
  if (cudaSetDevice(ctx->device) != cudaSuccess)
    return set_error(ctx, HAR_CUDA_ERR_CUDA, "ep_create: cudaSetDevice failed");
  ncclUniqueId id;
  memcpy(&id, unique_id, sizeof(id));
  har_cuda_ep *ep = new har_cuda_ep;
  ep->world = world;
  ep->rank = rank;
  ep->device = ctx->device;
  ep->op_timeout_ms = timeout_ms;
  bool ok = cudaStreamCreateWithFlags(&ep->cs, cudaStreamNonBlocking) == cudaSuccess;
  for (int i = 0; i < 4 && ok; ++i)
    ok = cudaEventCreateWithFlags(&ep->ev[i], cudaEventDisableTiming) == cudaSuccess;
  if (!ok) {
    har_cuda_ep_free(ep);
    return set_error(ctx, HAR_CUDA_ERR_CUDA, "ep_create: stream or event creation failed");
  }
  ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
  config.blocking = 0;  // init and group calls return at once; nccl_settle bounds them
  ncclResult_t r = ncclCommInitRankConfig(&ep->comm, world, id, rank, &config);
  const int32_t st = ep->comm ? nccl_settle(ctx, &ep->comm, r, "ep_create: joining the communicator",
                                            timeout_ms)
                              : nccl_error(ctx, "ncclCommInitRankConfig", r);
  if (st) {
    har_cuda_ep_free(ep);  // an aborted communicator is already gone
    return st;
  }
  *out = ep;
  return HAR_CUDA_OK;
}

int32_t har_cuda_ep_create(har_cuda_ctx *ctx, const uint8_t *unique_id, size_t len, int32_t world,
                           int32_t rank, har_cuda_ep **out) {
  return har_cuda_ep_create_timeout(ctx, unique_id, len, world, rank, 300000, out);
}

int32_t har_cuda_ep_abort(har_cuda_ep *ep) {
  if (!ep) return HAR_CUDA_ERR_ARG;
  if (ep->comm) {
    ncclCommAbort(ep->comm);
    ep->comm = nullptr;
  }
  return HAR_CUDA_OK;
}

int32_t har_cuda_ep_free(har_cuda_ep *ep) {
  if (!ep) return HAR_CUDA_OK;
  cudaSetDevice(ep->device);
  if (ep->buf) {
    cudaDeviceSynchronize();
    cudaFree(ep->buf);
  }
  if (ep->comm) {
    // finalize (non-blocking: poll, bounded), then destroy; a communicator
    // whose finalize does not settle is aborted instead
    ncclResult_t r = ncclCommFinalize(ep->comm);
    const auto t0 = std::chrono::steady_clock::now();
    ncclResult_t state = r;
    while (r == ncclSuccess || r == ncclInProgress) {
      if (ncclCommGetAsyncError(ep->comm, &state) != ncclSuccess || state != ncclInProgress) break;
      if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(ep->op_timeout_ms)) break;
      std::this_thread::sleep_for(std::chrono::microseconds(100));
    }
    if ((r == ncclSuccess || r == ncclInProgress) && state == ncclSuccess)
      ncclCommDestroy(ep->comm);
    else
      ncclCommAbort(ep->comm);
  }
  for (int i = 0; i < 4; ++i)
    if (ep->ev[i]) cudaEventDestroy(ep->ev[i]);
  if (ep->cs) {
    cudaStreamSynchronize(ep->cs);
    cudaStreamDestroy(ep->cs);
  }
  delete ep;
  return HAR_CUDA_OK;
}

int32_t har_cuda_ep_plan(har_cuda_ctx *ctx, const float *x_dev, int64_t H, int64_t T, int32_t k,
                         const int32_t *ids_dev, const float *weights_dev, int32_t E, int32_t world,
                         float *sx_dev, int32_t *sids_dev, float *sw_dev) {
  if (!ctx) return HAR_CUDA_ERR_ARG;
  if (!x_dev || !ids_dev || !weights_dev || !sx_dev || !sids_dev || !sw_dev)
    return set_error(ctx, HAR_CUDA_ERR_ARG, "ep_plan: null pointer");
  if (world < 1 || E < world || E % world || k <= 0 || k > E || T < 0 || H <= 0 || H % 4 ||
      (int64_t)world * T > INT32_MAX || (int64_t)world * T * k > ((int64_t)1 << 24))
    return set_error(ctx, HAR_CUDA_ERR_GEOMETRY,
                     "ep_plan: need world | E, 0 < k <= E, H a multiple of 4, world*T*k <= 2^24");
  if (((uintptr_t)x_dev & 15u) || ((uintptr_t)sx_dev & 15u))
    return set_error(ctx, HAR_CUDA_ERR_ARG, "ep_plan: x and sx must be 16-byte aligned");
  if (cudaSetDevice(ctx->device) != cudaSuccess)
    return set_error(ctx, HAR_CUDA_ERR_CUDA, "ep_plan: cudaSetDevice failed");
  if (T == 0) return HAR_CUDA_OK;
  prof_begin(ctx);
  ep_plan_kernel<<<(unsigned)(world * T), 128, 0, ctx->stream>>>(x_dev, (int)H, ids_dev, weights_dev,
                                                                (int)T, k, E, E / world, sx_dev,
                                                                sids_dev, sw_dev, -1, ctx->d_status);
  return check_launch(ctx, "ep_plan_kernel");
}

int32_t har_cuda_ep_combine(har_cuda_ctx *ctx, const float *x_dev, int64_t H, int64_t T,
                            int32_t world, const float *shared_dev, const float *back_dev,
                            uint32_t flags, float *y_dev) {
  if (!ctx) return HAR_CUDA_ERR_ARG;
  if (!x_dev || !back_dev || !y_dev) return set_error(ctx, HAR_CUDA_ERR_ARG, "ep_combine: null pointer");
  if (world < 1 || T < 0 || T > INT32_MAX || H <= 0 || H > INT32_MAX)
    return set_error(ctx, HAR_CUDA_ERR_GEOMETRY, "ep_combine: need world >= 1, T >= 0, H > 0");
  if (flags & ~HAR_CUDA_MOE_ADD_RESIDUAL)
    return set_error(ctx, HAR_CUDA_ERR_ARG, "ep_combine: only HAR_CUDA_MOE_ADD_RESIDUAL applies");
  if (cudaSetDevice(ctx->device) != cudaSuccess)
    return set_error(ctx, HAR_CUDA_ERR_CUDA, "ep_combine: cudaSetDevice failed");
  if (T == 0) return HAR_CUDA_OK;
  prof_begin(ctx);
  ep_combine_kernel<<<(unsigned)T, 256, 0, ctx->stream>>>(x_dev, (int)H, (int)T, world, shared_dev,
                                                         back_dev,
                                                         (flags & HAR_CUDA_MOE_ADD_RESIDUAL) ? 1 : 0,
                                                         y_dev);
  return check_launch(ctx, "ep_combine_kernel");
}

int32_t har_cuda_ep_moe_ffn(har_cuda_ctx *ctx, har_cuda_ep *ep, const har_cuda_moe_layer *local,
                            const har_cuda_moe_layer *shared, const float *gate_inp_dev,
                            const float *x_dev, int64_t T, int32_t k, const int32_t *ids_dev,
                            const float *weights_dev, float *y_dev, uint32_t flags) {
  int32_t st = ep_check(ctx, ep, local, shared, T, k, flags);
  if (st) return st;
  if (!x_dev || !ids_dev || !weights_dev || !y_dev)
    return set_error(ctx, HAR_CUDA_ERR_ARG, "ep_moe_ffn: null pointer");
  if (cudaSetDevice(ctx->device) != cudaSuccess)
    return set_error(ctx, HAR_CUDA_ERR_CUDA, "ep_moe_ffn: cudaSetDevice failed");
  if (T == 0) return HAR_CUDA_OK;
  return ep_layer(ctx, ep, local, shared, gate_inp_dev, x_dev, T, k, ids_dev, weights_dev, y_dev,
                  flags);
}

int32_t har_cuda_ep_moe_stack(har_cuda_ctx *ctx, har_cuda_ep *ep,
                              const har_cuda_moe_layer *const *local_layers,
                              const har_cuda_moe_layer *const *shared_layers,
                              const float *const *gate_inp_devs, int32_t L, const float *x_dev,
                              int64_t T, int32_t k, const int32_t *ids_dev,
                              const float *weights_dev, float *y_dev, uint32_t flags) {
  if (!ctx) return HAR_CUDA_ERR_ARG;
  if (!local_layers || L <= 0) return set_error(ctx, HAR_CUDA_ERR_ARG, "ep_moe_stack: no layers");
  if (!x_dev || !ids_dev || !weights_dev || !y_dev)
    return set_error(ctx, HAR_CUDA_ERR_ARG, "ep_moe_stack: null pointer");
  for (int l = 0; l < L; ++l) {
    int32_t st = ep_check(ctx, ep, local_layers[l], shared_layers ? shared_layers[l] : nullptr, T,
                          k, flags);
    if (st) return st;
    if (local_layers[l]->H != local_layers[0]->H)
      return set_error(ctx, HAR_CUDA_ERR_GEOMETRY, "ep_moe_stack: layers differ in hidden size");
  }
  if (cudaSetDevice(ctx->device) != cudaSuccess)
    return set_error(ctx, HAR_CUDA_ERR_CUDA, "ep_moe_stack: cudaSetDevice failed");
  if (T == 0) return HAR_CUDA_OK;
  const float *in = x_dev;
  for (int l = 0; l < L; ++l) {
    int32_t st = ep_layer(ctx, ep, local_layers[l], shared_layers ? shared_layers[l] : nullptr,
                          gate_inp_devs ? gate_inp_devs[l] : nullptr, in, T, k,
                          ids_dev + (size_t)l * T * k, weights_dev + (size_t)l * T * k, y_dev,
                          flags);
    if (st) return st;
    in = y_dev;  // every read of a layer's input precedes the combine that writes y
  }
  return HAR_CUDA_OK;
}

}  // extern "C"
