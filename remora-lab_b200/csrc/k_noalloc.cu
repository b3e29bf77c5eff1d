// k_noalloc.cu — har_cuda_moe_ffn_noalloc: the MoE FFN layer without any
// device allocation, for callers that cannot call cudaMalloc.
//
// Who needs it: serving runtimes that reserve a GPU's memory up front for
// their own pools (expert slots, KV pages) and hand the library only the
// buffers of a call, so an allocation behind their back either fails or
// breaks their accounting; and decode loops that cannot afford the
// device-wide synchronisation cudaMalloc/cudaFree may imply.  The regular
// har_cuda_moe_ffn grows a per-context scratch arena with cudaMalloc on first
// use; this variant runs the same kernels on a fixed scratch region that
// lives in the library image instead.
//
// The scratch is a file-scope __device__ array of HAR_CUDA_NOALLOC_SCRATCH_BYTES
// (32 MiB).  Every GPU that loads this library's device code holds it until
// the process exits.  Host code cannot use the array's name as a device
// address (on the host it names a stand-in object), so the first call in
// each CUDA context looks up the real address with cudaGetSymbolAddress while
// that context is current, and caches it per context; that first call should
// be made before any stream capture.  All calls on a device share the array and
// it keeps the last call's contents: the kernels write every scratch word
// before reading it, so nothing needs clearing between calls, but calls that
// overlap on the GPU (two streams or two contexts on one device) race on it
// and must be serialised by the caller.
#include <cuda.h>

#include <mutex>
#include <vector>

#include "har_internal.cuh"

namespace har {

static __device__ __align__(256) uint8_t noalloc_scratch[HAR_CUDA_NOALLOC_SCRATCH_BYTES];

// Cached device addresses of noalloc_scratch, one per CUDA context.  The key
// is the current driver context, not the device index: after a
// cudaDeviceReset (or under a context other than the device's primary one)
// the array lives at a new address, which a per-device cache would miss.
struct NoallocEntry {
  CUcontext cu;
  void *ptr;
};
static std::vector<NoallocEntry> noalloc_cache;
static std::mutex noalloc_mu;

using CtxGetCurrentFn = CUresult (*)(CUcontext *);

static CtxGetCurrentFn ctx_get_current_fn() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (CtxGetCurrentFn)p;
    cudaGetLastError();
  });
  return fn;
}

// Device address of noalloc_scratch in the current context (ctx->device is
// current; looked up once per context).
static int32_t noalloc_scratch_ptr(har_cuda_ctx *ctx, uint8_t **out) {
  CtxGetCurrentFn get = ctx_get_current_fn();
  CUcontext cu = nullptr;
  // cudaFree(0) makes the runtime bind the device's context to this thread
  if (!get || cudaFree(0) != cudaSuccess || get(&cu) != CUDA_SUCCESS || !cu) {
    cudaGetLastError();
    return set_error(ctx, HAR_CUDA_ERR_CUDA, "moe_ffn_noalloc: no current CUDA context");
  }
  std::lock_guard<std::mutex> lock(noalloc_mu);
  for (const NoallocEntry &e : noalloc_cache)
    if (e.cu == cu) {
      *out = (uint8_t *)e.ptr;
      return HAR_CUDA_OK;
    }
  void *p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, noalloc_scratch);
  if (e != cudaSuccess || !p) {
    cudaGetLastError();
    return set_error(ctx, HAR_CUDA_ERR_CUDA,
                     std::string("moe_ffn_noalloc: cudaGetSymbolAddress failed: ") +
                         cudaGetErrorString(e));
  }
  noalloc_cache.push_back({cu, p});
  *out = (uint8_t *)p;
  return HAR_CUDA_OK;
}

}  // namespace har

using namespace har;

extern "C" int32_t har_cuda_moe_ffn_noalloc(har_cuda_ctx *ctx, const har_cuda_moe_layer *layer,
                                            const float *x_dev, int64_t T, int32_t k,
                                            const int32_t *ids_dev, const float *weights_dev,
                                            float *y_dev, uint32_t flags) {
  int32_t st = check_moe_args(ctx, layer, T, k, flags);
  if (st != HAR_CUDA_OK) return st;
  if (T == 0) return HAR_CUDA_OK;
  if (!x_dev || !ids_dev || !weights_dev || !y_dev)
    return set_error(ctx, HAR_CUDA_ERR_ARG, "moe_ffn_noalloc: null pointer");
  const size_t need = moe_scratch_bytes(ctx, layer, T, k, flags);
  if (need > (size_t)HAR_CUDA_NOALLOC_SCRATCH_BYTES)
    return set_error(ctx, HAR_CUDA_ERR_GEOMETRY,
                     "moe_ffn_noalloc: this call needs " + std::to_string(need) +
                         " bytes of scratch; the static scratch holds " +
                         std::to_string((size_t)HAR_CUDA_NOALLOC_SCRATCH_BYTES) +
                         " (use fewer tokens per call, or har_cuda_moe_ffn)");
  cudaError_t e = cudaSetDevice(ctx->device);
  if (e != cudaSuccess)
    return set_error(ctx, HAR_CUDA_ERR_CUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(e));
  uint8_t *scratch = nullptr;
  st = noalloc_scratch_ptr(ctx, &scratch);
  if (st != HAR_CUDA_OK) return st;
  return run_moe_ffn_in(ctx, layer, x_dev, T, k, ids_dev, weights_dev, y_dev, flags, scratch);
}
