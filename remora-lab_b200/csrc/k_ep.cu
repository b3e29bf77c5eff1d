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
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

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
  // Peer-memory exchange: every rank's window (flags, staged token rows, the
  // partial sums it computes) is mapped into every other rank's address space
  // by CUDA IPC, and the rows move by loads over NVLink instead of NCCL.
  int p2p = 0;          // requested (har_cuda_ep_set_p2p, opt-in); the windows are set up on first use
  int p2p_state = 0;    // 0 not set up, 1 mapped on every rank, -1 some rank could not (NCCL only)
  void *win = nullptr;  // this rank's window
  size_t win_bytes = 0;
  void **peer = nullptr;      // host: every rank's window in this process (peer[rank] = win)
  void **peer_dev = nullptr;  // the same array on the device
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

// ---- peer-memory exchange -------------------------------------------------
// Window of rank r (the same layout on every rank):
//   u32 flags[2G + 1]: dispatch[d] / ret[d] = the last epoch rank d posted to
//                      r, then r's own epoch (layers so far);
//   staged rows:       x[T][H], ids[T][k], w[T][k] of r's tokens;
//   part[G*T][H]:      r's partial sums for the rows it received (row d*T + t
//                      = token t of rank d).
// Per layer: r stages its rows, bumps its epoch e and posts e to every rank's
// dispatch[r]; each rank pulls the rows that have an expert of its own (its
// wait: dispatch[d] >= e for the rank d it reads); runs its experts into
// part; posts e to every rank's ret[r]; and sums its tokens' partials pulled
// from the ranks that hold one of their experts.  A rank rewrites its staged
// rows (next layer) only after its combine saw every rank's ret flag, i.e.
// after every rank finished pulling them, and its part only after every rank
// staged the next layer, i.e. after they all combined: no buffer is reused
// while a peer may still read it.  Waits poll with acquire loads, sleep
// between polls and give up after the communicator's timeout
// (DEV_ERR_TIMEOUT, reported by the next status check); the ranks are
// separate GPUs, so a waiting kernel never holds up the kernel it waits for.

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait for *flag >= e (epochs compared modulo 2^32).  False on
// timeout (flagged in status) or when another wait of the call already gave up.
__device__ bool ep_wait_flag(const uint32_t *flag, uint32_t e, uint64_t limit_ns, int *status) {
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0;; ++i) {
    if ((int32_t)(ld_acquire_sys(flag) - e) >= 0) return true;
    if ((i & 31u) == 31u) {
      if (*(volatile int *)status & DEV_ERR_TIMEOUT) return false;
      if (globaltimer_ns() - t0 > limit_ns) {
        atomicOr(status, DEV_ERR_TIMEOUT);
        return false;
      }
    }
    __nanosleep(64);
  }
}

// This rank's tokens into its window: x rows, ids (checked) and weights.
__global__ void __launch_bounds__(128) ep_stage_kernel(const float *__restrict__ x, int H,
                                                       const int32_t *__restrict__ ids,
                                                       const float *__restrict__ w, int k, int E,
                                                       float *__restrict__ sx, int32_t *__restrict__ sids,
                                                       float *__restrict__ sw, int *status) {
  const int64_t t = blockIdx.x;
  for (int j = threadIdx.x; j < k; j += blockDim.x) {
    const int e = ids[t * k + j];
    if (e < 0 || e >= E) atomicOr(status, DEV_ERR_BOUNDS);
    sids[t * k + j] = e;
    sw[t * k + j] = w[t * k + j];
  }
  const float4 *src = reinterpret_cast<const float4 *>(x + t * H);
  float4 *dst = reinterpret_cast<float4 *>(sx + t * H);
  for (int i = threadIdx.x; i < H / 4; i += blockDim.x) dst[i] = src[i];
}

// Post this rank's epoch to slot `which` (0 dispatch, 1 ret) of every rank's
// flags; bump = advance the epoch first (once per layer).  Peer data is read
// with ld.global.cv (fetched again, never served from a cached line).
__global__ void ep_post_kernel(uint32_t *own, void *const *peer, int which, int rank, int G, int bump) {
  if (threadIdx.x != 0) return;
  uint32_t e = own[2 * G];
  if (bump) own[2 * G] = ++e;
  __threadfence_system();  // the rows and partial sums written before this launch, then the flags
  for (int d = 0; d < G; ++d) st_release_sys(reinterpret_cast<uint32_t *>(peer[d]) + which * G + rank, e);
}

// Row (d, t) of this rank's input: token t of rank d, pulled from d's window
// when one of its slots has an expert here (always for d == keep: the shared
// expert reads this rank's own rows); its slots as local ids (-1 elsewhere).
__global__ void __launch_bounds__(128) ep_pull_kernel(const uint32_t *own, void *const *peer,
                                                      size_t off_x, size_t off_ids, size_t off_w, int T,
                                                      int H, int k, int El, int rank, int G, int keep,
                                                      float *__restrict__ rx, int32_t *__restrict__ rids,
                                                      float *__restrict__ rw, uint64_t wait_ns, int *status) {
  const int d = blockIdx.x / T, t = blockIdx.x % T;
  const int64_t row = (int64_t)d * T + t;
  __shared__ int ok_s, any;
  if (threadIdx.x == 0) {
    ok_s = ep_wait_flag(own + d, own[2 * G], wait_ns, status) ? 1 : 0;
    if (ok_s) __threadfence_system();
    any = 0;
  }
  __syncthreads();
  if (!ok_s) {  // the wait gave up: the row is left out (empty slots), the error is reported
    for (int j = threadIdx.x; j < k; j += blockDim.x) {
      rids[row * k + j] = -1;
      rw[row * k + j] = 0.0f;
    }
    return;
  }
  const uint8_t *pb = reinterpret_cast<const uint8_t *>(peer[d]);
  const int32_t *pids = reinterpret_cast<const int32_t *>(pb + off_ids) + (int64_t)t * k;
  const float *pw = reinterpret_cast<const float *>(pb + off_w) + (int64_t)t * k;
  for (int j = threadIdx.x; j < k; j += blockDim.x) {
    const int e = __ldcv(pids + j);
    int loc = -1;
    if (e >= 0 && e < El * G && e / El == rank) {
      loc = e - rank * El;
      any = 1;
    }
    rids[row * k + j] = loc;
    rw[row * k + j] = loc >= 0 ? __ldcv(pw + j) : 0.0f;
  }
  __syncthreads();
  if (!any && d != keep) return;
  const float4 *src = reinterpret_cast<const float4 *>(pb + off_x) + (int64_t)t * (H / 4);
  float4 *dst = reinterpret_cast<float4 *>(rx + row * H);
  for (int i = threadIdx.x; i < H / 4; i += blockDim.x) dst[i] = __ldcv(src + i);
}

// y[t] = (x[t] with the residual flag) + the partial sums of token t from the
// ranks that hold one of its experts (and this rank's, which holds the shared
// expert), in rank order: the NCCL path's sum with its zero terms left out.
__global__ void __launch_bounds__(256) ep_combine_pull_kernel(const float *x, int H, int T, int G, int El,
                                                              int rank, const int32_t *__restrict__ ids,
                                                              int k, const uint32_t *own, void *const *peer,
                                                              size_t off_part, int residual, float *y,
                                                              uint64_t wait_ns, int *status) {
  const int t = blockIdx.x;
  __shared__ int ok_s;
  __shared__ uint32_t has;
  if (threadIdx.x == 0) {
    const uint32_t e = own[2 * G];
    bool ok = true;
    for (int d = 0; ok && d < G; ++d) ok = ep_wait_flag(own + G + d, e, wait_ns, status);
    if (ok) __threadfence_system();
    ok_s = ok ? 1 : 0;
    uint32_t m = 1u << rank;
    for (int j = 0; j < k; ++j) {
      const int ex = ids[(int64_t)t * k + j];
      if (ex >= 0 && ex < El * G) m |= 1u << (ex / El);
    }
    has = m;
  }
  __syncthreads();
  if (!ok_s) return;
  const uint32_t m = has;
  const int64_t prow = ((int64_t)rank * T + t) * H;
  for (int h = threadIdx.x; h < H; h += blockDim.x) {
    const int64_t i = (int64_t)t * H + h;
    float acc = residual ? x[i] : 0.0f;
    for (int d = 0; d < G; ++d)
      if ((m >> d) & 1u)
        acc = __fadd_rn(acc, __ldcv(reinterpret_cast<const float *>(
                                        reinterpret_cast<const uint8_t *>(peer[d]) + off_part) + prow + h));
    y[i] = acc;
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

// ---- peer-memory windows ----------------------------------------------------
struct WinLayout {
  size_t x, ids, w, part, total;  // the flags sit at offset 0
};

WinLayout win_layout(int G, int64_t T, int k, int64_t H) {
  WinLayout W;
  size_t off = 0;
  auto take = [&](size_t b) { size_t o = off; off += al256(b); return o; };
  take(4 * (size_t)(2 * G + 1));
  W.x = take(4 * (size_t)T * H);
  W.ids = take(4 * (size_t)T * k);
  W.w = take(4 * (size_t)T * k);
  W.part = take(4 * (size_t)G * T * H);
  W.total = off;
  return W;
}

// Wait for the exchange stream's work (a setup collective), bounded by the
// communicator's timeout: on expiry the communicator is aborted, which ends
// the NCCL kernel that waits for the missing rank.
int32_t ep_stream_wait(har_cuda_ctx *ctx, har_cuda_ep *ep, const char *what) {
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    const cudaError_t q = cudaStreamQuery(ep->cs);
    if (q == cudaSuccess) return HAR_CUDA_OK;
    if (q != cudaErrorNotReady)
      return set_error(ctx, HAR_CUDA_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(q));
    if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(ep->op_timeout_ms)) {
      if (ep->comm) ncclCommAbort(ep->comm);
      ep->comm = nullptr;
      return set_error(ctx, HAR_CUDA_ERR_TIMEOUT, std::string(what) + " did not complete; the communicator was aborted");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

// A one-int all-reduce (min) over the ranks on the exchange stream: the
// agreement (and barrier) step of the window setup and release.
int32_t ep_agree(har_cuda_ctx *ctx, har_cuda_ep *ep, int32_t *dev_int, int32_t mine, int32_t *out,
                 const char *what) {
  if (!ep->comm) return set_error(ctx, HAR_CUDA_ERR_NOT_INIT, "ep: no communicator");
  if (cudaMemcpyAsync(dev_int, &mine, 4, cudaMemcpyHostToDevice, ep->cs) != cudaSuccess)
    return set_error(ctx, HAR_CUDA_ERR_CUDA, std::string(what) + ": copy failed");
  int32_t st = nccl_settle(ctx, &ep->comm, ncclAllReduce(dev_int, dev_int, 1, ncclInt32, ncclMin, ep->comm, ep->cs),
                           what, ep->op_timeout_ms);
  if (st) return st;
  if (cudaMemcpyAsync(out, dev_int, 4, cudaMemcpyDeviceToHost, ep->cs) != cudaSuccess)
    return set_error(ctx, HAR_CUDA_ERR_CUDA, std::string(what) + ": copy failed");
  return ep_stream_wait(ctx, ep, what);
}

// A barrier over the ranks without a context (for har_cuda_ep_free), bounded
// by the communicator's timeout.  False when it did not complete.
bool ep_barrier_raw(har_cuda_ep *ep) {
  if (!ep->comm) return false;
  int32_t *d = nullptr;
  if (cudaMalloc(&d, 4) != cudaSuccess) return false;
  cudaMemsetAsync(d, 0, 4, ep->cs);
  const ncclResult_t r = ncclAllReduce(d, d, 1, ncclInt32, ncclMin, ep->comm, ep->cs);
  bool ok = r == ncclSuccess || r == ncclInProgress;
  const auto t0 = std::chrono::steady_clock::now();
  while (ok) {
    ncclResult_t state = ncclSuccess;
    if (ncclCommGetAsyncError(ep->comm, &state) != ncclSuccess || (state != ncclSuccess && state != ncclInProgress)) {
      ok = false;
      break;
    }
    if (state == ncclSuccess) {
      const cudaError_t q = cudaStreamQuery(ep->cs);
      if (q == cudaSuccess) break;
      if (q != cudaErrorNotReady) {
        ok = false;
        break;
      }
    }
    if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(ep->op_timeout_ms)) {
      ok = false;
      break;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
  if (ok) cudaFree(d);  // else the all-reduce may still hold it
  return ok;
}

// Close the imported windows of the other ranks.
void ep_p2p_unmap(har_cuda_ep *ep) {
  if (ep->peer)
    for (int d = 0; d < ep->world; ++d)
      if (d != ep->rank && ep->peer[d]) cudaIpcCloseMemHandle(ep->peer[d]);
  delete[] ep->peer;
  ep->peer = nullptr;
  if (ep->peer_dev) cudaFree(ep->peer_dev);
  ep->peer_dev = nullptr;
}

// Collective: unmap the peers' windows, then free this rank's own once every
// rank has unmapped it (a barrier).  Without a working communicator the own
// window is left allocated: a peer may still have it mapped.
int32_t ep_p2p_release(har_cuda_ctx *ctx, har_cuda_ep *ep, int32_t *dev_int) {
  if (!ep->win && !ep->peer) return HAR_CUDA_OK;
  cudaStreamSynchronize(ctx->stream);  // this rank's kernels that read the windows (their waits are bounded)
  ep_p2p_unmap(ep);
  int32_t all = 0, st = HAR_CUDA_ERR_NOT_INIT;
  if (ep->comm && dev_int) st = ep_agree(ctx, ep, dev_int, 1, &all, "ep: window release");
  if (!st && ep->win) cudaFree(ep->win);
  ep->win = nullptr;
  ep->win_bytes = 0;
  ep->p2p_state = 0;
  return st;
}

// Collective on first use (and when a call needs a larger window): allocate
// this rank's window, exchange IPC handles and PCI locations over NCCL, map
// every other rank's window.  The peer path is taken only when every rank
// mapped every window and the ranks sit on distinct GPUs (a waiting kernel
// must never share its GPU with the kernel it waits for); otherwise all ranks
// keep the NCCL path.  Needs a call outside graph capture first.
struct EpPeerRec {
  cudaIpcMemHandle_t h;
  int32_t domain, bus, dev, ok;
};

int32_t ep_p2p_setup(har_cuda_ctx *ctx, har_cuda_ep *ep, size_t bytes) {
  if (ep->p2p_state < 0 || (ep->p2p_state == 1 && ep->win_bytes >= bytes)) return HAR_CUDA_OK;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(ctx->stream, &cap);
  if (cap != cudaStreamCaptureStatusNone)
    return set_error(ctx, HAR_CUDA_ERR_UNSUPPORTED,
                     "ep: the peer-memory windows are set up by a call outside graph capture "
                     "(run the same shape once before capturing)");
  const int G = ep->world;
  uint8_t *tmp = nullptr;  // G records, then one int
  if (cudaMalloc(&tmp, (size_t)G * sizeof(EpPeerRec) + 16) != cudaSuccess)
    return set_error(ctx, HAR_CUDA_ERR_OOM, "ep: window setup buffer");
  int32_t *dint = reinterpret_cast<int32_t *>(tmp + (size_t)G * sizeof(EpPeerRec));
  int32_t st = ep_p2p_release(ctx, ep, dint);
  if (st) {
    cudaFree(tmp);
    return st;
  }
  EpPeerRec me{};
  // the zeroed flags are in place before any rank finishes the handle
  // exchange below (same stream), so no peer's first post can be overwritten
  me.ok = G <= 32 && cudaMalloc(&ep->win, bytes) == cudaSuccess;
  if (me.ok)
    me.ok = cudaMemsetAsync(ep->win, 0, bytes, ep->cs) == cudaSuccess &&
            cudaIpcGetMemHandle(&me.h, ep->win) == cudaSuccess;
  cudaDeviceGetAttribute(&me.domain, cudaDevAttrPciDomainId, ctx->device);
  cudaDeviceGetAttribute(&me.bus, cudaDevAttrPciBusId, ctx->device);
  cudaDeviceGetAttribute(&me.dev, cudaDevAttrPciDeviceId, ctx->device);
  cudaGetLastError();
  std::vector<EpPeerRec> all(G);
  uint8_t *slot = tmp + (size_t)ep->rank * sizeof(EpPeerRec);
  if (cudaMemcpyAsync(slot, &me, sizeof(me), cudaMemcpyHostToDevice, ep->cs) != cudaSuccess) {
    cudaFree(tmp);
    return set_error(ctx, HAR_CUDA_ERR_CUDA, "ep: window setup copy failed");
  }
  st = nccl_settle(ctx, &ep->comm, ncclAllGather(slot, tmp, sizeof(EpPeerRec), ncclUint8, ep->comm, ep->cs),
                   "ep: window handle exchange", ep->op_timeout_ms);
  if (!st && cudaMemcpyAsync(all.data(), tmp, (size_t)G * sizeof(EpPeerRec), cudaMemcpyDeviceToHost, ep->cs) != cudaSuccess)
    st = set_error(ctx, HAR_CUDA_ERR_CUDA, "ep: window setup copy failed");
  if (!st) st = ep_stream_wait(ctx, ep, "ep: window handle exchange");
  if (st) {
    cudaFree(tmp);
    return st;
  }
  // the same records on every rank, so every rank takes the same decision here
  bool ok = true;
  for (int d = 0; d < G; ++d) {
    ok = ok && all[d].ok;
    for (int c = 0; c < d; ++c)
      if (all[c].domain == all[d].domain && all[c].bus == all[d].bus && all[c].dev == all[d].dev) ok = false;
  }
  int32_t mapped = 0;
  if (ok) {
    ep->peer = new void *[G]();
    mapped = 1;
    for (int d = 0; d < G; ++d) {
      if (d == ep->rank) {
        ep->peer[d] = ep->win;
        continue;
      }
      // peer access to rank d's GPU checked and enabled here, so that a pair
      // without it (or a device out of peer connections) keeps every rank on
      // NCCL instead of failing at the first load
      char bus[32];
      snprintf(bus, sizeof bus, "%04x:%02x:%02x.0", all[d].domain, all[d].bus, all[d].dev);
      int pdev = -1, can = 0;
      if (cudaDeviceGetByPCIBusId(&pdev, bus) != cudaSuccess ||
          cudaDeviceCanAccessPeer(&can, ctx->device, pdev) != cudaSuccess || !can) {
        mapped = 0;
        continue;
      }
      const cudaError_t pe = cudaDeviceEnablePeerAccess(pdev, 0);
      if (pe != cudaSuccess && pe != cudaErrorPeerAccessAlreadyEnabled) {
        mapped = 0;
        continue;
      }
      cudaGetLastError();
      if (cudaIpcOpenMemHandle(&ep->peer[d], all[d].h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        ep->peer[d] = nullptr;
        mapped = 0;
      }
    }
    cudaGetLastError();
    if (mapped) {
      mapped = cudaMalloc(&ep->peer_dev, (size_t)G * sizeof(void *)) == cudaSuccess &&
               cudaMemcpy(ep->peer_dev, ep->peer, (size_t)G * sizeof(void *), cudaMemcpyHostToDevice) == cudaSuccess;
    }
  }
  int32_t every = 0;
  st = ep_agree(ctx, ep, dint, mapped, &every, "ep: window mapping");
  if (!st && !every) {
    // some rank could not map: everyone unmaps, then frees its own window
    // after a barrier, and the layers stay on NCCL
    st = ep_p2p_release(ctx, ep, dint);
    ep->p2p_state = -1;
  } else if (!st) {
    ep->win_bytes = bytes;
    ep->p2p_state = 1;
  }
  cudaFree(tmp);
  return st;
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
  const WinLayout W = win_layout(G, T, k, H);
  if (ep->p2p && G > 1 && (st = ep_p2p_setup(ctx, ep, W.total))) return st;
  const bool peer_path = ep->p2p && ep->p2p_state == 1;
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
  const int residual = (flags & HAR_CUDA_MOE_ADD_RESIDUAL) ? 1 : 0;
  if (peer_path) {
    // stage -> post -> pull -> experts -> post -> combine, all on ctx->stream
    uint8_t *wb = (uint8_t *)ep->win;
    uint32_t *own = reinterpret_cast<uint32_t *>(wb);
    void *const *pd = reinterpret_cast<void *const *>(ep->peer_dev);
    float *wpart = reinterpret_cast<float *>(wb + W.part);
    const uint64_t wait_ns = (uint64_t)ep->op_timeout_ms * 1000000ull;  // the communicator's bound
    prof_begin(ctx);
    ep_stage_kernel<<<(unsigned)T, 128, 0, ctx->stream>>>(x, (int)H, ids, w, k, E, reinterpret_cast<float *>(wb + W.x),
                                                         reinterpret_cast<int32_t *>(wb + W.ids),
                                                         reinterpret_cast<float *>(wb + W.w), ctx->d_status);
    if ((st = check_launch(ctx, "ep_stage_kernel"))) return st;
    prof_begin(ctx);
    ep_post_kernel<<<1, 32, 0, ctx->stream>>>(own, pd, 0, ep->rank, G, 1);
    if ((st = check_launch(ctx, "ep_post_kernel"))) return st;
    prof_begin(ctx);
    ep_pull_kernel<<<(unsigned)(G * T), 128, 0, ctx->stream>>>(own, pd, W.x, W.ids, W.w, (int)T, (int)H, k, El,
                                                               ep->rank, G, shared ? ep->rank : -1, rx, rids, rw,
                                                               wait_ns, ctx->d_status);
    if ((st = check_launch(ctx, "ep_pull_kernel"))) return st;
    if ((st = run_moe_ffn_range(ctx, lay, rx, (int64_t)G * T, k, rids, rw, wpart, lmode,
                                (uint8_t *)ctx->scratch, shared ? (int64_t)ep->rank * T : 0,
                                shared ? T : 0)))
      return st;
    prof_begin(ctx);
    ep_post_kernel<<<1, 32, 0, ctx->stream>>>(own, pd, 1, ep->rank, G, 0);
    if ((st = check_launch(ctx, "ep_post_kernel"))) return st;
    prof_begin(ctx);
    ep_combine_pull_kernel<<<(unsigned)T, 256, 0, ctx->stream>>>(x, (int)H, (int)T, G, El, ep->rank, ids, k, own, pd,
                                                                W.part, residual, y, wait_ns, ctx->d_status);
    return check_launch(ctx, "ep_combine_pull_kernel");
  }
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
  ep_combine_kernel<<<(unsigned)T, 256, 0, ctx->stream>>>(x, (int)H, (int)T, G, nullptr, back, residual, y);
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

int32_t har_cuda_ep_set_p2p(har_cuda_ep *ep, int32_t on) {
  if (!ep) return HAR_CUDA_ERR_ARG;
  ep->p2p = on ? 1 : 0;
  return HAR_CUDA_OK;
}

int32_t har_cuda_ep_exchange_mode(const har_cuda_ep *ep) {
  if (!ep) return HAR_CUDA_ERR_ARG;
  if (!ep->p2p) return 0;
  return ep->p2p_state;
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
  if (ep->win || ep->peer) {
    // collective like the window setup: unmap the peers' windows, then free
    // this rank's once every rank has unmapped it; without that barrier (no
    // communicator, or a rank gone) the window stays allocated
    cudaDeviceSynchronize();
    ep_p2p_unmap(ep);
    if (ep_barrier_raw(ep) && ep->win) cudaFree(ep->win);
    ep->win = nullptr;
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
