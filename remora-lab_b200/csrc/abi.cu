// abi.cu — C ABI entry points of libhar_cuda.so (declared in include/har_cuda.h):
// context, error reporting, weight handles, argument checking.  Kernels live
// in the k_*.cu files; this file validates geometry the way the reference's
// expert_matvec does (har/crates/har-demo/src/bin/har-native-qwen35moe.rs:632-662)
// and turns every failure into a status code instead of a panic.
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <chrono>
#include <thread>

#include "har_internal.cuh"

namespace har {

int32_t set_error(har_cuda_ctx *ctx, int32_t code, const std::string &msg) {
  if (ctx) ctx->last_error = msg;
  return code;
}

void prof_begin(har_cuda_ctx *ctx) {
  if (!ctx->prof_on) return;
  cudaEvent_t a;
  if (cudaEventCreate(&a) != cudaSuccess) return;
  cudaEventRecord(a, ctx->stream);
  ctx->prof_pending = a;
}

int32_t check_launch(har_cuda_ctx *ctx, const char *what) {
  cudaError_t e = cudaGetLastError();
  if (ctx->prof_on && ctx->prof_pending) {
    cudaEvent_t b;
    if (cudaEventCreate(&b) == cudaSuccess) {
      cudaEventRecord(b, ctx->stream);
      ctx->prof.push_back({what, ctx->prof_pending, b});
    } else {
      cudaEventDestroy(ctx->prof_pending);
    }
    ctx->prof_pending = nullptr;
  }
  if (e != cudaSuccess)
    return set_error(ctx, HAR_CUDA_ERR_CUDA,
                     std::string(what) + ": " + cudaGetErrorString(e));
  ctx->launches += 1;
  return HAR_CUDA_OK;
}

static void prof_clear(har_cuda_ctx *ctx) {
  for (auto &r : ctx->prof) {
    cudaEventDestroy(r.a);
    cudaEventDestroy(r.b);
  }
  ctx->prof.clear();
  if (ctx->prof_pending) cudaEventDestroy(ctx->prof_pending);
  ctx->prof_pending = nullptr;
}

int32_t ensure_scratch(har_cuda_ctx *ctx, size_t bytes) {
  if (bytes <= ctx->scratch_bytes) return HAR_CUDA_OK;
  // Growing frees the old arena: wait for work that may still use it.
  if (ctx->scratch) {
    cudaStreamSynchronize(ctx->stream);
    cudaFree(ctx->scratch);
    ctx->scratch = nullptr;
    ctx->scratch_bytes = 0;
  }
  size_t sz = (bytes + (1u << 20) - 1) & ~((size_t)(1u << 20) - 1);
  if (cudaMalloc(&ctx->scratch, sz) != cudaSuccess) {
    cudaGetLastError();
    return set_error(ctx, HAR_CUDA_ERR_OOM,
                     "scratch allocation of " + std::to_string(sz) + " bytes failed");
  }
  ctx->scratch_bytes = sz;
  ++ctx->epoch;
  return HAR_CUDA_OK;
}

static int32_t ensure_pinned(har_cuda_ctx *ctx, size_t bytes) {
  if (bytes <= ctx->host_pinned_bytes) return HAR_CUDA_OK;
  if (ctx->host_pinned) {
    cudaStreamSynchronize(ctx->stream);
    cudaFreeHost(ctx->host_pinned);
    ctx->host_pinned = nullptr;
    ctx->host_pinned_bytes = 0;
  }
  size_t sz = (bytes + (1u << 20) - 1) & ~((size_t)(1u << 20) - 1);
  if (cudaMallocHost(&ctx->host_pinned, sz) != cudaSuccess) {
    cudaGetLastError();
    return set_error(ctx, HAR_CUDA_ERR_OOM, "pinned host staging allocation failed");
  }
  ctx->host_pinned_bytes = sz;
  ++ctx->epoch;
  return HAR_CUDA_OK;
}

static int32_t ensure_io(har_cuda_ctx *ctx, size_t bytes) {
  if (bytes <= ctx->io_dev_bytes) return HAR_CUDA_OK;
  if (ctx->io_dev) {
    cudaStreamSynchronize(ctx->stream);
    cudaFree(ctx->io_dev);
    ctx->io_dev = nullptr;
    ctx->io_dev_bytes = 0;
  }
  size_t sz = (bytes + (1u << 20) - 1) & ~((size_t)(1u << 20) - 1);
  if (cudaMalloc(&ctx->io_dev, sz) != cudaSuccess) {
    cudaGetLastError();
    return set_error(ctx, HAR_CUDA_ERR_OOM, "device staging allocation failed");
  }
  ctx->io_dev_bytes = sz;
  ++ctx->epoch;
  return HAR_CUDA_OK;
}

static int32_t use_device(har_cuda_ctx *ctx) {
  cudaError_t e = cudaSetDevice(ctx->device);
  if (e != cudaSuccess)
    return set_error(ctx, HAR_CUDA_ERR_CUDA,
                     std::string("cudaSetDevice: ") + cudaGetErrorString(e));
  return HAR_CUDA_OK;
}

static int32_t check_weights(har_cuda_ctx *ctx, const har_cuda_weights *w, const char *name,
                             int32_t type = GGML_Q4_K) {
  if (!w) return set_error(ctx, HAR_CUDA_ERR_ARG, std::string(name) + " is null");
  if (!w->dev) return set_error(ctx, HAR_CUDA_ERR_NOT_INIT, std::string(name) + " has no data");
  if (w->device != ctx->device)
    return set_error(ctx, HAR_CUDA_ERR_ARG, std::string(name) + " lives on another device");
  if (w->type != type)
    return set_error(ctx, HAR_CUDA_ERR_UNSUPPORTED,
                     std::string(name) + " has GGML type " + std::to_string(w->type) +
                         ", this call needs type " + std::to_string(type));
  return HAR_CUDA_OK;
}

}  // namespace har

using namespace har;

#define HAR_TRY(expr)                       \
  do {                                      \
    int32_t _st = (expr);                   \
    if (_st != HAR_CUDA_OK) return _st;     \
  } while (0)

extern "C" {

int32_t har_cuda_abi_version(void) { return HAR_CUDA_ABI_VERSION; }

int32_t har_cuda_ctx_create(int32_t device, har_cuda_ctx **out) {
  if (!out) return HAR_CUDA_ERR_ARG;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
    cudaGetLastError();
    return HAR_CUDA_ERR_CUDA;  // no device: fail closed, no CPU fallback
  }
  if (device < 0 || device >= n) return HAR_CUDA_ERR_ARG;
  if (cudaSetDevice(device) != cudaSuccess) return HAR_CUDA_ERR_CUDA;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return HAR_CUDA_ERR_CUDA;
  if (prop.major != 10) return HAR_CUDA_ERR_UNSUPPORTED;  // built for sm_100a only
  har_cuda_ctx *ctx = new har_cuda_ctx();
  ctx->device = device;
  ctx->num_sms = prop.multiProcessorCount;
  if (cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMalloc(&ctx->d_status, sizeof(int) * 4) != cudaSuccess ||
      cudaMemset(ctx->d_status, 0, sizeof(int) * 4) != cudaSuccess) {
    cudaGetLastError();
    delete ctx;
    return HAR_CUDA_ERR_CUDA;
  }
  ctx->stream = ctx->own_stream;
  *out = ctx;
  return HAR_CUDA_OK;
}

int32_t har_cuda_ctx_destroy(har_cuda_ctx *ctx) {
  if (!ctx) return HAR_CUDA_ERR_ARG;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  prof_clear(ctx);
  if (ctx->host_graph.exec) cudaGraphExecDestroy(ctx->host_graph.exec);
  if (ctx->scratch) cudaFree(ctx->scratch);
  if (ctx->host_pinned) cudaFreeHost(ctx->host_pinned);
  if (ctx->io_dev) cudaFree(ctx->io_dev);
  if (ctx->d_status) cudaFree(ctx->d_status);
  if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
  delete ctx;
  return HAR_CUDA_OK;
}

int32_t har_cuda_last_error(const har_cuda_ctx *ctx, char *buf, size_t len) {
  if (!ctx || !buf || len == 0) return HAR_CUDA_ERR_ARG;
  size_t n = ctx->last_error.size() < len - 1 ? ctx->last_error.size() : len - 1;
  memcpy(buf, ctx->last_error.data(), n);
  buf[n] = '\0';
  return HAR_CUDA_OK;
}

int32_t har_cuda_ctx_set_stream(har_cuda_ctx *ctx, void *cuda_stream) {
  if (!ctx) return HAR_CUDA_ERR_ARG;
  ctx->stream = cuda_stream ? (cudaStream_t)cuda_stream : ctx->own_stream;
  return HAR_CUDA_OK;
}

int32_t har_cuda_ctx_set_tc_min_tokens(har_cuda_ctx *ctx, int32_t min_tokens) {
  if (!ctx) return HAR_CUDA_ERR_ARG;
  if (min_tokens < 0) return har::set_error(ctx, HAR_CUDA_ERR_ARG, "set_tc_min_tokens: negative");
  ctx->tc_min_tokens = min_tokens;
  return HAR_CUDA_OK;
}

int64_t har_cuda_launch_count(const har_cuda_ctx *ctx) { return ctx ? ctx->launches : -1; }

int32_t har_cuda_profile_begin(har_cuda_ctx *ctx) {
  if (!ctx) return HAR_CUDA_ERR_ARG;
  prof_clear(ctx);
  ctx->prof_on = true;
  return HAR_CUDA_OK;
}

int32_t har_cuda_profile_end(har_cuda_ctx *ctx, char *names, size_t names_len, float *ms,
                             int64_t cap, int64_t *count) {
  if (!ctx || !count) return HAR_CUDA_ERR_ARG;
  ctx->prof_on = false;
  if (cudaSetDevice(ctx->device) != cudaSuccess || cudaStreamSynchronize(ctx->stream) != cudaSuccess) {
    cudaGetLastError();
    prof_clear(ctx);
    return set_error(ctx, HAR_CUDA_ERR_CUDA, "profile_end: stream synchronisation failed");
  }
  std::string all;
  int64_t n = 0;
  for (auto &r : ctx->prof) {
    if (n < cap) {
      float t = 0.0f;
      cudaEventElapsedTime(&t, r.a, r.b);
      if (ms) ms[n] = t;
      all += r.name;
      all += '\n';
    }
    ++n;
  }
  if (names && names_len) {
    size_t m = all.size() < names_len - 1 ? all.size() : names_len - 1;
    memcpy(names, all.data(), m);
    names[m] = '\0';
  }
  *count = n < cap ? n : cap;
  prof_clear(ctx);
  return HAR_CUDA_OK;
}

int32_t har_cuda_synchronize(har_cuda_ctx *ctx, int64_t timeout_ms) {
  if (!ctx) return HAR_CUDA_ERR_ARG;
  HAR_TRY(use_device(ctx));
  cudaEvent_t ev;
  if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess)
    return set_error(ctx, HAR_CUDA_ERR_CUDA, "cudaEventCreate failed");
  cudaEventRecord(ev, ctx->stream);
  auto t0 = std::chrono::steady_clock::now();
  int32_t st = HAR_CUDA_OK;
  for (;;) {
    cudaError_t q = cudaEventQuery(ev);
    if (q == cudaSuccess) break;
    if (q != cudaErrorNotReady) {
      st = set_error(ctx, HAR_CUDA_ERR_CUDA, std::string("stream error: ") + cudaGetErrorString(q));
      break;
    }
    auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                  std::chrono::steady_clock::now() - t0).count();
    if (timeout_ms >= 0 && ms > timeout_ms) {
      st = set_error(ctx, HAR_CUDA_ERR_TIMEOUT, "stream did not finish within the deadline");
      break;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
  cudaEventDestroy(ev);
  if (st != HAR_CUDA_OK) return st;
  int word = 0;
  if (cudaMemcpyAsync(&word, ctx->d_status, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream) !=
          cudaSuccess ||
      cudaStreamSynchronize(ctx->stream) != cudaSuccess)
    return set_error(ctx, HAR_CUDA_ERR_CUDA, "status readback failed");
  if (word != 0) {
    cudaMemsetAsync(ctx->d_status, 0, sizeof(int), ctx->stream);
    cudaStreamSynchronize(ctx->stream);
    std::string why = "a kernel reported device error word " + std::to_string(word);
    if (word & DEV_ERR_TIMEOUT) why += " (a bounded wait ran out)";
    if (word & DEV_ERR_BOUNDS) why += " (an expert id out of range)";
    if (word & DEV_ERR_RANGE)
      why += " (a value beyond the tensor-core path's f16 range -- |x|, a sub-block sum or a SwiGLU "
             "output >= 65520 -- or an unrepresentable Q4_K block: run it with HAR_CUDA_MOE_FORCE_GEMV)";
    return set_error(ctx, word & DEV_ERR_TIMEOUT ? HAR_CUDA_ERR_TIMEOUT : HAR_CUDA_ERR_DEVICE, why);
  }
  return HAR_CUDA_OK;
}

static int32_t make_weights(har_cuda_ctx *ctx, int32_t type, int64_t E, int64_t N, int64_t K,
                            har_cuda_weights **out) {
  if (!ctx || !out) return HAR_CUDA_ERR_ARG;
  *out = nullptr;
  if (!ggml_block_bytes(type))
    return set_error(ctx, HAR_CUDA_ERR_UNSUPPORTED,
                     "weights: GGML type " + std::to_string(type) +
                         " (supported: 11 Q3_K, 12 Q4_K, 14 Q6_K)");
  if (E <= 0 || N <= 0 || K <= 0)
    return set_error(ctx, HAR_CUDA_ERR_GEOMETRY, "weights: E, N and K must be positive");
  if (K % QK != 0)
    return set_error(ctx, HAR_CUDA_ERR_GEOMETRY,
                     "weights: K=" + std::to_string(K) + " is not a multiple of 256");
  har_cuda_weights *w = new har_cuda_weights();
  w->E = E;
  w->N = N;
  w->K = K;
  w->type = type;
  w->row_bytes = K / QK * ggml_block_bytes(type);
  w->expert_bytes = w->row_bytes * N;
  w->device = ctx->device;
  *out = w;
  return HAR_CUDA_OK;
}

int32_t har_cuda_weights_upload_q4k(har_cuda_ctx *ctx, const void *host_bytes, int64_t E,
                                    int64_t N, int64_t K, har_cuda_weights **out) {
  return har_cuda_weights_upload(ctx, GGML_Q4_K, host_bytes, E, N, K, out);
}

int32_t har_cuda_weights_wrap_q4k(har_cuda_ctx *ctx, const void *dev_bytes, int64_t E,
                                  int64_t N, int64_t K, har_cuda_weights **out) {
  return har_cuda_weights_wrap(ctx, GGML_Q4_K, dev_bytes, E, N, K, out);
}

int32_t har_cuda_weights_upload(har_cuda_ctx *ctx, int32_t ggml_type, const void *host_bytes,
                                int64_t E, int64_t N, int64_t K, har_cuda_weights **out) {
  HAR_TRY(make_weights(ctx, ggml_type, E, N, K, out));
  har_cuda_weights *w = *out;
  if (!host_bytes) {
    delete w;
    *out = nullptr;
    return set_error(ctx, HAR_CUDA_ERR_ARG, "weights_upload: host_bytes is null");
  }
  HAR_TRY(use_device(ctx));
  size_t bytes = (size_t)(w->expert_bytes * E);
  void *d = nullptr;
  if (cudaMalloc(&d, bytes) != cudaSuccess) {
    cudaGetLastError();
    delete w;
    *out = nullptr;
    return set_error(ctx, HAR_CUDA_ERR_OOM, "weights_upload: cudaMalloc failed");
  }
  if (cudaMemcpyAsync(d, host_bytes, bytes, cudaMemcpyHostToDevice, ctx->stream) != cudaSuccess ||
      cudaStreamSynchronize(ctx->stream) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(d);
    delete w;
    *out = nullptr;
    return set_error(ctx, HAR_CUDA_ERR_CUDA, "weights_upload: copy failed");
  }
  w->dev = (const uint8_t *)d;
  w->owned = true;
  return HAR_CUDA_OK;
}

int32_t har_cuda_weights_wrap(har_cuda_ctx *ctx, int32_t ggml_type, const void *dev_bytes,
                              int64_t E, int64_t N, int64_t K, har_cuda_weights **out) {
  HAR_TRY(make_weights(ctx, ggml_type, E, N, K, out));
  if (!dev_bytes || ((uintptr_t)dev_bytes & 15u)) {
    delete *out;
    *out = nullptr;
    return set_error(ctx, HAR_CUDA_ERR_ARG, "weights_wrap: pointer null or not 16-byte aligned");
  }
  (*out)->dev = (const uint8_t *)dev_bytes;
  (*out)->owned = false;
  return HAR_CUDA_OK;
}

int32_t har_cuda_weights_free(har_cuda_weights *w) {
  if (!w) return HAR_CUDA_ERR_ARG;
  if (w->owned && w->dev) {
    cudaSetDevice(w->device);
    cudaFree((void *)w->dev);
  }
  delete w;
  return HAR_CUDA_OK;
}

const void *har_cuda_weights_device_ptr(const har_cuda_weights *w) { return w ? w->dev : nullptr; }

int32_t har_cuda_q8k_quantize(har_cuda_ctx *ctx, const float *x_dev, int64_t M, int64_t K,
                              void *out_dev) {
  if (!ctx) return HAR_CUDA_ERR_ARG;
  if (!x_dev || !out_dev) return set_error(ctx, HAR_CUDA_ERR_ARG, "q8k_quantize: null pointer");
  if (M < 0 || K <= 0 || K % QK != 0)
    return set_error(ctx, HAR_CUDA_ERR_GEOMETRY, "q8k_quantize: K must be a positive multiple of 256");
  if (M == 0) return HAR_CUDA_OK;
  HAR_TRY(use_device(ctx));
  return launch_q8k_quantize(ctx, x_dev, M, K, (uint8_t *)out_dev);
}

int32_t har_cuda_q4k_gemv(har_cuda_ctx *ctx, const har_cuda_weights *w, int64_t expert,
                          const void *x_dev, int32_t act_kind, int64_t M, float *y_dev) {
  if (!ctx) return HAR_CUDA_ERR_ARG;
  HAR_TRY(check_weights(ctx, w, "q4k_gemv: weights"));
  if (!x_dev || !y_dev) return set_error(ctx, HAR_CUDA_ERR_ARG, "q4k_gemv: null pointer");
  if (expert < 0 || expert >= w->E)
    return set_error(ctx, HAR_CUDA_ERR_ARG, "expert " + std::to_string(expert) +
                                                " exceeds model expert count " + std::to_string(w->E));
  if (act_kind != HAR_CUDA_ACT_F32 && act_kind != HAR_CUDA_ACT_Q8K)
    return set_error(ctx, HAR_CUDA_ERR_ARG, "q4k_gemv: unknown act_kind");
  if (M < 0) return set_error(ctx, HAR_CUDA_ERR_GEOMETRY, "q4k_gemv: negative M");
  if (M == 0) return HAR_CUDA_OK;
  HAR_TRY(use_device(ctx));
  return launch_gemv(ctx, w, expert, x_dev, act_kind, M, y_dev);
}

int32_t har_cuda_q3k_gemv(har_cuda_ctx *ctx, const har_cuda_weights *w, int64_t expert,
                          const float *x_dev, int64_t M, float *y_dev) {
  if (!ctx) return HAR_CUDA_ERR_ARG;
  HAR_TRY(check_weights(ctx, w, "q3k_gemv: weights", GGML_Q3_K));
  if (!x_dev || !y_dev) return set_error(ctx, HAR_CUDA_ERR_ARG, "q3k_gemv: null pointer");
  if (expert < 0 || expert >= w->E)
    return set_error(ctx, HAR_CUDA_ERR_ARG, "q3k_gemv: expert " + std::to_string(expert) +
                                                " out of range [0, " + std::to_string(w->E) + ")");
  if (M < 0 || M > ((int64_t)1 << 19))
    return set_error(ctx, HAR_CUDA_ERR_GEOMETRY, "q3k_gemv: need 0 <= M <= 2^19");
  if (((uintptr_t)x_dev & 15u) || ((uintptr_t)y_dev & 3u))
    return set_error(ctx, HAR_CUDA_ERR_ARG, "q3k_gemv: x must be 16-byte aligned, y 4-byte");
  if (M == 0) return HAR_CUDA_OK;
  HAR_TRY(use_device(ctx));
  return launch_q3k_gemv(ctx, w, expert, x_dev, M, y_dev);
}

int32_t har_cuda_q6k_gemv(har_cuda_ctx *ctx, const har_cuda_weights *w, int64_t expert,
                          const float *x_dev, int64_t M, float *y_dev) {
  if (!ctx) return HAR_CUDA_ERR_ARG;
  HAR_TRY(check_weights(ctx, w, "q6k_gemv: weights", GGML_Q6_K));
  if (!x_dev || !y_dev) return set_error(ctx, HAR_CUDA_ERR_ARG, "q6k_gemv: null pointer");
  if (expert < 0 || expert >= w->E)
    return set_error(ctx, HAR_CUDA_ERR_ARG, "q6k_gemv: expert " + std::to_string(expert) +
                                                " out of range [0, " + std::to_string(w->E) + ")");
  if (M < 0 || M > ((int64_t)1 << 19))
    return set_error(ctx, HAR_CUDA_ERR_GEOMETRY, "q6k_gemv: need 0 <= M <= 2^19");
  if (((uintptr_t)x_dev & 15u) || ((uintptr_t)y_dev & 3u))
    return set_error(ctx, HAR_CUDA_ERR_ARG, "q6k_gemv: x must be 16-byte aligned, y 4-byte");
  if (M == 0) return HAR_CUDA_OK;
  HAR_TRY(use_device(ctx));
  return launch_q6k_gemv(ctx, w, expert, x_dev, M, y_dev);
}

int32_t har_cuda_route_topk(har_cuda_ctx *ctx, const float *logits_dev, int64_t T, int32_t E,
                            int32_t k, int32_t *ids_dev, float *weights_dev) {
  if (!ctx) return HAR_CUDA_ERR_ARG;
  if (!logits_dev || !ids_dev || !weights_dev)
    return set_error(ctx, HAR_CUDA_ERR_ARG, "route_topk: null pointer");
  if (T < 0 || E <= 0 || k <= 0 || k > E || k > 32 || E > 8192)
    return set_error(ctx, HAR_CUDA_ERR_GEOMETRY,
                     "route_topk: need 0 < k <= min(E, 32) and E <= 8192");
  if (T == 0) return HAR_CUDA_OK;
  HAR_TRY(use_device(ctx));
  return launch_route_topk(ctx, logits_dev, T, E, k, ids_dev, weights_dev);
}

int32_t har_cuda_router_logits(har_cuda_ctx *ctx, const float *gate_inp_dev, int32_t E,
                               int64_t H, const float *x_dev, int64_t T, float *logits_dev) {
  if (!ctx) return HAR_CUDA_ERR_ARG;
  if (!gate_inp_dev || !x_dev || !logits_dev)
    return set_error(ctx, HAR_CUDA_ERR_ARG, "router_logits: null pointer");
  if (T < 0 || E <= 0 || H <= 0 || H > ((int64_t)1 << 24) || T > ((int64_t)1 << 21))
    return set_error(ctx, HAR_CUDA_ERR_GEOMETRY,
                     "router_logits: need E > 0, 0 < H <= 2^24 and 0 <= T <= 2^21");
  if (T == 0) return HAR_CUDA_OK;
  HAR_TRY(use_device(ctx));
  return launch_router_logits(ctx, gate_inp_dev, E, (int)H, x_dev, T, logits_dev);
}

int32_t har_cuda_route(har_cuda_ctx *ctx, const float *gate_inp_dev, int32_t E, int64_t H,
                       const float *x_dev, int64_t T, int32_t k, int32_t *ids_dev,
                       float *weights_dev) {
  if (!ctx) return HAR_CUDA_ERR_ARG;
  if (!gate_inp_dev || !x_dev || !ids_dev || !weights_dev)
    return set_error(ctx, HAR_CUDA_ERR_ARG, "route: null pointer");
  if (T < 0 || E <= 0 || k <= 0 || k > E || k > 32 || E > 8192 || H <= 0 ||
      H > ((int64_t)1 << 24) || T > ((int64_t)1 << 21))
    return set_error(ctx, HAR_CUDA_ERR_GEOMETRY,
                     "route: need 0 < k <= min(E, 32), E <= 8192, 0 < H <= 2^24, T <= 2^21");
  if (T == 0) return HAR_CUDA_OK;
  HAR_TRY(use_device(ctx));
  // logits live in the scratch arena only until route_topk has read them
  HAR_TRY(ensure_scratch(ctx, sizeof(float) * (size_t)T * (size_t)E));
  float *logits = static_cast<float *>(ctx->scratch);
  bool fused = false;  // decode batches: logits and top-k in one launch
  HAR_TRY(launch_route_fused(ctx, gate_inp_dev, E, (int)H, x_dev, T, k, logits, ids_dev,
                             weights_dev, &fused));
  if (fused) return HAR_CUDA_OK;
  HAR_TRY(launch_router_logits(ctx, gate_inp_dev, E, (int)H, x_dev, T, logits));
  return launch_route_topk(ctx, logits, T, E, k, ids_dev, weights_dev);
}

int32_t har_cuda_group_by_expert(har_cuda_ctx *ctx, const int32_t *ids_dev, int64_t T,
                                 int32_t k, int32_t E, int32_t *counts_dev,
                                 int32_t *offsets_dev, int32_t *order_dev) {
  if (!ctx) return HAR_CUDA_ERR_ARG;
  if (!ids_dev || !counts_dev || !offsets_dev || !order_dev)
    return set_error(ctx, HAR_CUDA_ERR_ARG, "group_by_expert: null pointer");
  if (T < 0 || k <= 0 || E <= 0 || E > 2048 || T * k > (int64_t)1 << 24)
    return set_error(ctx, HAR_CUDA_ERR_GEOMETRY, "group_by_expert: E <= 2048, T*k <= 2^24");
  HAR_TRY(use_device(ctx));
  // scratch: inv[T*k], then the multi-CTA sort's segment counts (if any)
  const size_t inv_words = ((size_t)(T * k) + 63) & ~(size_t)63;
  const size_t gw = group_scratch_words(T * k, E);
  HAR_TRY(ensure_scratch(ctx, sizeof(int32_t) * (inv_words + gw + 1)));
  int32_t *inv = (int32_t *)ctx->scratch;
  return launch_group(ctx, ids_dev, T, k, E, counts_dev, offsets_dev, order_dev, inv,
                      gw ? inv + inv_words : nullptr);
}

int32_t har_cuda_moe_layer_create(har_cuda_ctx *ctx, const har_cuda_weights *gate,
                                  const har_cuda_weights *up, const har_cuda_weights *down,
                                  const har_cuda_weights *sh_gate,
                                  const har_cuda_weights *sh_up,
                                  const har_cuda_weights *sh_down,
                                  const float *sh_gate_inp_dev, har_cuda_moe_layer **out) {
  if (!ctx || !out) return HAR_CUDA_ERR_ARG;
  *out = nullptr;
  HAR_TRY(check_weights(ctx, gate, "moe_layer: gate"));
  HAR_TRY(check_weights(ctx, up, "moe_layer: up"));
  HAR_TRY(check_weights(ctx, down, "moe_layer: down"));
  const int64_t E = gate->E, I = gate->N, H = gate->K;
  if (up->E != E || up->N != I || up->K != H || down->E != E || down->N != H || down->K != I)
    return set_error(ctx, HAR_CUDA_ERR_GEOMETRY,
                     "moe_layer: gate/up must be [E][I][H], down [E][H][I]");
  const bool any_sh = sh_gate || sh_up || sh_down;
  if (any_sh) {
    HAR_TRY(check_weights(ctx, sh_gate, "moe_layer: shared gate"));
    HAR_TRY(check_weights(ctx, sh_up, "moe_layer: shared up"));
    HAR_TRY(check_weights(ctx, sh_down, "moe_layer: shared down"));
    if (sh_gate->E != 1 || sh_gate->N != I || sh_gate->K != H || sh_up->E != 1 ||
        sh_up->N != I || sh_up->K != H || sh_down->E != 1 || sh_down->N != H ||
        sh_down->K != I)
      return set_error(ctx, HAR_CUDA_ERR_GEOMETRY,
                       "moe_layer: shared expert must be one expert of the routed shape");
  } else if (sh_gate_inp_dev) {
    return set_error(ctx, HAR_CUDA_ERR_ARG, "moe_layer: shared gate row without shared expert");
  }
  if (I % QK != 0 || H % QK != 0)
    return set_error(ctx, HAR_CUDA_ERR_GEOMETRY, "moe_layer: H and I must be multiples of 256");
  static std::atomic<uint64_t> next_gen{1};
  har_cuda_moe_layer *l = new har_cuda_moe_layer();
  l->gen = next_gen.fetch_add(1);
  l->gate = gate;
  l->up = up;
  l->down = down;
  l->sh_gate = sh_gate;
  l->sh_up = sh_up;
  l->sh_down = sh_down;
  l->sh_gate_inp = sh_gate_inp_dev;
  l->E = E;
  l->H = H;
  l->I = I;
  // Weight tensor maps for the tensor-core path (H and I multiples of 128).
  if (H % 128 == 0 && I % 128 == 0) {
    auto wmap = [&](TmaDesc *m, const har_cuda_weights *w) {
      return encode_tmap_2d(ctx, m, w->dev, 1, (uint64_t)(w->E * w->N), (uint64_t)w->row_bytes,
                            (uint64_t)w->row_bytes, 128, Q4K_BYTES, false);
    };
    int32_t st = wmap(&l->map_gate, gate);
    if (!st) st = wmap(&l->map_up, up);
    if (!st) st = wmap(&l->map_down, down);
    if (!st && any_sh) st = wmap(&l->map_sh_gate, sh_gate);
    if (!st && any_sh) st = wmap(&l->map_sh_up, sh_up);
    if (!st && any_sh) st = wmap(&l->map_sh_down, sh_down);
    if (st) {
      delete l;
      return st;
    }
    l->tc_maps = true;
  }
  *out = l;
  return HAR_CUDA_OK;
}

int32_t har_cuda_moe_layer_free(har_cuda_moe_layer *layer) {
  if (!layer) return HAR_CUDA_ERR_ARG;
  const int device = layer->gate ? layer->gate->device : 0;  // before the weights go
  for (har_cuda_weights *w : layer->owned)
    if (w) har_cuda_weights_free(w);
  if (layer->owned_dev) {
    cudaSetDevice(device);
    cudaFree(layer->owned_dev);
  }
  delete layer;
  return HAR_CUDA_OK;
}

}  // extern "C"

int32_t har::check_moe_args(har_cuda_ctx *ctx, const har_cuda_moe_layer *layer, int64_t T,
                            int32_t k, uint32_t flags) {
  if (!ctx) return HAR_CUDA_ERR_ARG;
  if (!layer) return set_error(ctx, HAR_CUDA_ERR_ARG, "moe_ffn: layer is null");
  if (T < 0 || k <= 0 || k > layer->E)
    return set_error(ctx, HAR_CUDA_ERR_GEOMETRY, "moe_ffn: need T >= 0 and 0 < k <= E");
  if (layer->E > 2048 || T * (int64_t)k > ((int64_t)1 << 24))
    return set_error(ctx, HAR_CUDA_ERR_GEOMETRY, "moe_ffn: E <= 2048 and T*k <= 2^24");
  if ((flags & HAR_CUDA_MOE_FORCE_GEMV) && (flags & HAR_CUDA_MOE_FORCE_TC))
    return set_error(ctx, HAR_CUDA_ERR_ARG, "moe_ffn: FORCE_GEMV and FORCE_TC are exclusive");
  if ((flags & HAR_CUDA_MOE_ACT_Q8K) && (flags & HAR_CUDA_MOE_FORCE_TC))
    return set_error(ctx, HAR_CUDA_ERR_UNSUPPORTED,
                     "moe_ffn: the tensor-core path has no Q8_K activation mode");
  if (flags & ~0x7Fu) return set_error(ctx, HAR_CUDA_ERR_ARG, "moe_ffn: unknown flag bits");
  if ((flags & HAR_CUDA_MOE_DECODE) &&
      (flags & (HAR_CUDA_MOE_ACT_Q8K | HAR_CUDA_MOE_FORCE_TC | HAR_CUDA_MOE_TC_F16W | HAR_CUDA_MOE_EMPTY_SLOTS)))
    return set_error(ctx, HAR_CUDA_ERR_ARG,
                     "moe_ffn: HAR_CUDA_MOE_DECODE runs f32 activations on CUDA cores: not with ACT_Q8K, "
                     "FORCE_TC, TC_F16W or EMPTY_SLOTS");
  return HAR_CUDA_OK;
}

extern "C" {

int32_t har_cuda_moe_ffn(har_cuda_ctx *ctx, const har_cuda_moe_layer *layer,
                         const float *x_dev, int64_t T, int32_t k, const int32_t *ids_dev,
                         const float *weights_dev, float *y_dev, uint32_t flags) {
  HAR_TRY(check_moe_args(ctx, layer, T, k, flags));
  if (T == 0) return HAR_CUDA_OK;
  if (!x_dev || !ids_dev || !weights_dev || !y_dev)
    return set_error(ctx, HAR_CUDA_ERR_ARG, "moe_ffn: null pointer");
  HAR_TRY(use_device(ctx));
  return run_moe_ffn(ctx, layer, x_dev, T, k, ids_dev, weights_dev, y_dev, flags);
}

int32_t har_cuda_routed_moe(har_cuda_ctx *ctx, const har_cuda_moe_layer *layer,
                            const float *gate_inp_dev, const float *x_dev, int64_t T, int32_t k,
                            int32_t *ids_dev, float *weights_dev, float *y_dev, uint32_t flags) {
  HAR_TRY(check_moe_args(ctx, layer, T, k, flags));
  if (flags & HAR_CUDA_MOE_EMPTY_SLOTS)
    return set_error(ctx, HAR_CUDA_ERR_ARG, "routed_moe: EMPTY_SLOTS is for the EP exchange only");
  if (T == 0) return HAR_CUDA_OK;
  if (!gate_inp_dev) gate_inp_dev = layer->router;  // the layer's own (GGUF) router
  if (!gate_inp_dev)
    return set_error(ctx, HAR_CUDA_ERR_ARG, "routed_moe: no router (argument null, layer has none)");
  if (!x_dev || !ids_dev || !weights_dev || !y_dev)
    return set_error(ctx, HAR_CUDA_ERR_ARG, "routed_moe: null pointer");
  HAR_TRY(har_cuda_route(ctx, gate_inp_dev, (int32_t)layer->E, layer->H, x_dev, T, k, ids_dev,
                         weights_dev));
  return run_moe_ffn(ctx, layer, x_dev, T, k, ids_dev, weights_dev, y_dev, flags);
}

int32_t har_cuda_routed_moe_stack(har_cuda_ctx *ctx, const har_cuda_moe_layer *const *layers,
                                  int32_t L, const float *const *gate_inp_devs,
                                  const float *x_dev, int64_t T, int32_t k, int32_t *ids_dev,
                                  float *weights_dev, float *y_dev, uint32_t flags) {
  if (!ctx) return HAR_CUDA_ERR_ARG;
  if (!layers || L <= 0) return set_error(ctx, HAR_CUDA_ERR_ARG, "routed_moe_stack: no layers");
  for (int l = 0; l < L; ++l) {
    HAR_TRY(check_moe_args(ctx, layers[l], T, k, flags));
    if (layers[l]->H != layers[0]->H)
      return set_error(ctx, HAR_CUDA_ERR_GEOMETRY, "routed_moe_stack: layers of different H");
    if (!(gate_inp_devs && gate_inp_devs[l]) && !layers[l]->router)
      return set_error(ctx, HAR_CUDA_ERR_ARG,
                       "routed_moe_stack: layer " + std::to_string(l) + " has no router");
  }
  if (flags & HAR_CUDA_MOE_EMPTY_SLOTS)
    return set_error(ctx, HAR_CUDA_ERR_ARG, "routed_moe_stack: EMPTY_SLOTS is for the EP exchange only");
  if (T == 0) return HAR_CUDA_OK;
  if (!x_dev || !ids_dev || !weights_dev || !y_dev)
    return set_error(ctx, HAR_CUDA_ERR_ARG, "routed_moe_stack: null pointer");
  HAR_TRY(use_device(ctx));
  const float *in = x_dev;
  for (int l = 0; l < L; ++l) {
    const float *gi = gate_inp_devs && gate_inp_devs[l] ? gate_inp_devs[l] : layers[l]->router;
    int32_t *ids = ids_dev + (size_t)l * T * k;
    float *w = weights_dev + (size_t)l * T * k;
    HAR_TRY(har_cuda_route(ctx, gi, (int32_t)layers[l]->E, layers[l]->H, in, T, k, ids, w));
    HAR_TRY(run_moe_ffn(ctx, layers[l], in, T, k, ids, w, y_dev, flags));
    in = y_dev;  // in-place chaining: the router and the layer read y before it is rewritten
  }
  return HAR_CUDA_OK;
}

int32_t har_cuda_moe_ffn_host(har_cuda_ctx *ctx, const har_cuda_moe_layer *layer,
                              const float *x_host, int64_t T, int32_t k,
                              const int32_t *ids_host, const float *weights_host,
                              float *y_host, uint32_t flags) {
  HAR_TRY(check_moe_args(ctx, layer, T, k, flags));
  if (T == 0) return HAR_CUDA_OK;
  if (!x_host || !ids_host || !weights_host || !y_host)
    return set_error(ctx, HAR_CUDA_ERR_ARG, "moe_ffn_host: null pointer");
  HAR_TRY(use_device(ctx));
  const size_t xb = sizeof(float) * (size_t)(T * layer->H);
  const size_t ib = sizeof(int32_t) * (size_t)(T * k);
  const size_t wb = sizeof(float) * (size_t)(T * k);
  auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
  const size_t total = al(xb) + al(ib) + al(wb) + al(xb);
  HAR_TRY(ensure_pinned(ctx, total));
  char *hp = (char *)ctx->host_pinned;
  memcpy(hp, x_host, xb);
  memcpy(hp + al(xb), ids_host, ib);
  memcpy(hp + al(xb) + al(ib), weights_host, wb);
  // Device inputs sit in their own grow-only buffer so run_moe_ffn may grow scratch.
  HAR_TRY(ensure_io(ctx, total));
  char *dp = (char *)ctx->io_dev;
  cudaMemcpyAsync(dp, hp, al(xb) + al(ib) + al(wb), cudaMemcpyHostToDevice, ctx->stream);
  int32_t st = run_moe_ffn(ctx, layer, (const float *)dp, T, k,
                           (const int32_t *)(dp + al(xb)), (const float *)(dp + al(xb) + al(ib)),
                           (float *)(dp + al(xb) + al(ib) + al(wb)), flags);
  if (st == HAR_CUDA_OK) {
    char *hy = hp + al(xb) + al(ib) + al(wb);
    cudaMemcpyAsync(hy, dp + al(xb) + al(ib) + al(wb), xb, cudaMemcpyDeviceToHost, ctx->stream);
    st = har_cuda_synchronize(ctx, 60000);
    if (st == HAR_CUDA_OK) memcpy(y_host, hy, xb);
  }
  return st;
}

int32_t har_cuda_moe_stack(har_cuda_ctx *ctx, const har_cuda_moe_layer *const *layers,
                           int32_t L, const float *x_dev, int64_t T, int32_t k,
                           const int32_t *ids_dev, const float *weights_dev, float *y_dev,
                           uint32_t flags) {
  if (!ctx) return HAR_CUDA_ERR_ARG;
  if (!layers || L <= 0) return set_error(ctx, HAR_CUDA_ERR_ARG, "moe_stack: no layers");
  if (!x_dev || !ids_dev || !weights_dev || !y_dev)
    return set_error(ctx, HAR_CUDA_ERR_ARG, "moe_stack: null pointer");
  for (int l = 0; l < L; ++l) {
    HAR_TRY(check_moe_args(ctx, layers[l], T, k, flags));
    if (layers[l]->H != layers[0]->H)
      return set_error(ctx, HAR_CUDA_ERR_GEOMETRY, "moe_stack: layers differ in hidden size");
  }
  if (T == 0) return HAR_CUDA_OK;
  HAR_TRY(use_device(ctx));
  const float *in = x_dev;
  for (int l = 0; l < L; ++l) {
    HAR_TRY(run_moe_ffn(ctx, layers[l], in, T, k, ids_dev + (size_t)l * T * k,
                        weights_dev + (size_t)l * T * k, y_dev, flags));
    in = y_dev;  // in-place chaining: run_moe_ffn reads x before it writes y
  }
  return HAR_CUDA_OK;
}

int32_t har_cuda_moe_stack_host(har_cuda_ctx *ctx, const har_cuda_moe_layer *const *layers,
                                int32_t L, const float *x_host, int64_t T, int32_t k,
                                const int32_t *ids_host, const float *weights_host,
                                float *y_host, uint32_t flags) {
  if (!ctx) return HAR_CUDA_ERR_ARG;
  if (!layers || L <= 0) return set_error(ctx, HAR_CUDA_ERR_ARG, "moe_stack_host: no layers");
  if (!x_host || !ids_host || !weights_host || !y_host)
    return set_error(ctx, HAR_CUDA_ERR_ARG, "moe_stack_host: null pointer");
  for (int l = 0; l < L; ++l) HAR_TRY(check_moe_args(ctx, layers[l], T, k, flags));
  if (T == 0) return HAR_CUDA_OK;
  HAR_TRY(use_device(ctx));
  auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
  const size_t xb = sizeof(float) * (size_t)(T * layers[0]->H);
  const size_t rb = sizeof(int32_t) * (size_t)(L * T * k);
  const size_t in_b = al(xb) + al(rb) + al(rb);
  HAR_TRY(ensure_pinned(ctx, in_b + al(xb)));
  HAR_TRY(ensure_io(ctx, in_b + al(xb)));
  char *hp = (char *)ctx->host_pinned, *dp = (char *)ctx->io_dev;
  memcpy(hp, x_host, xb);
  memcpy(hp + al(xb), ids_host, rb);
  memcpy(hp + al(xb) + al(rb), weights_host, rb);
  float *yd = (float *)(dp + in_b);
  // copy in, the stack, copy out: all device work of the call, on ctx->stream
  auto enqueue = [&]() -> int32_t {
    cudaMemcpyAsync(dp, hp, in_b, cudaMemcpyHostToDevice, ctx->stream);
    int32_t st = har_cuda_moe_stack(ctx, layers, L, (const float *)dp, T, k,
                                    (const int32_t *)(dp + al(xb)),
                                    (const float *)(dp + al(xb) + al(rb)), yd, flags);
    if (st != HAR_CUDA_OK) return st;
    cudaMemcpyAsync(hp + in_b, yd, xb, cudaMemcpyDeviceToHost, ctx->stream);
    return HAR_CUDA_OK;
  };
  // A call repeated with the same key (layers, shapes, flags, threshold,
  // stream, and no reallocation since) replays a CUDA graph of its device work:
  // the second such call captures it (by then every buffer has its size).
  auto &g = ctx->host_graph;
  std::vector<uint64_t> key((size_t)L);
  for (int l = 0; l < L; ++l) key[l] = layers[l]->gen;
  const bool same = g.layers == key && g.T == T && g.k == k && g.flags == flags &&
                    g.tc_min == ctx->tc_min_tokens && g.epoch == ctx->epoch && g.stream == ctx->stream;
  if (!same) {
    if (g.exec) cudaGraphExecDestroy(g.exec);
    g = har_cuda_ctx::HostGraph();
    g.layers = key;
    g.T = T;
    g.k = k;
    g.flags = flags;
    g.tc_min = ctx->tc_min_tokens;
    g.stream = ctx->stream;
  }
  g.epoch = ctx->epoch;
  // stream capture is not allowed on the legacy or per-thread default stream
  // (handles 0, 0x1, 0x2): there every call runs eagerly
  const bool capturable = (uintptr_t)ctx->stream > (uintptr_t)0x2;
  if (!g.exec && g.seen >= 1 && !ctx->prof_on && capturable) {
    cudaGraph_t graph = nullptr;
    bool ok = cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
    const int32_t st = ok ? enqueue() : HAR_CUDA_OK;
    ok = cudaStreamEndCapture(ctx->stream, &graph) == cudaSuccess && ok && st == HAR_CUDA_OK;
    if (ok && cudaGraphInstantiate(&g.exec, graph, 0) != cudaSuccess) g.exec = nullptr;
    if (graph) cudaGraphDestroy(graph);
    cudaGetLastError();  // a failed capture falls back to the eager path below
    if (g.epoch != ctx->epoch && g.exec) {  // the capture reallocated: not replayable
      cudaGraphExecDestroy(g.exec);
      g.exec = nullptr;
    }
  }
  ++g.seen;
  if (g.exec && !ctx->prof_on) {
    if (cudaGraphLaunch(g.exec, ctx->stream) != cudaSuccess)
      return set_error(ctx, HAR_CUDA_ERR_DEVICE, "moe_stack_host: graph launch failed");
  } else {
    HAR_TRY(enqueue());
  }
  // a device error word (HAR_CUDA_ERR_DEVICE) comes from a finished stream:
  // the results are copied out as computed and the status marks them invalid
  const int32_t st = har_cuda_synchronize(ctx, 600000);
  if (st == HAR_CUDA_OK || st == HAR_CUDA_ERR_DEVICE) memcpy(y_host, hp + in_b, xb);
  return st;
}

int32_t har_cuda_gen_q4k(har_cuda_ctx *ctx, void *dev_bytes, int64_t rows, int64_t K,
                         uint64_t seed, int64_t row0, float mean, float stdv) {
  if (!ctx) return HAR_CUDA_ERR_ARG;
  if (!dev_bytes) return set_error(ctx, HAR_CUDA_ERR_ARG, "gen_q4k: null pointer");
  if (rows < 0 || K <= 0 || K % QK != 0)
    return set_error(ctx, HAR_CUDA_ERR_GEOMETRY, "gen_q4k: K must be a positive multiple of 256");
  if (rows == 0) return HAR_CUDA_OK;
  HAR_TRY(use_device(ctx));
  return launch_gen_q4k(ctx, (uint8_t *)dev_bytes, rows, K, seed, row0, mean, stdv);
}

}  // extern "C"
