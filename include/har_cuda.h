/*
 * har_cuda.h — C ABI of the B200-native Q4_K MoE-FFN path (libhar_cuda.so).
 *
 * This is the drop-in boundary HAR's Rust runtime binds through a thin FFI
 * crate (har-cuda).  Every function is extern "C", takes plain pointers and
 * sizes, and returns an int32 status: 0 = OK, negative = error (see
 * HAR_CUDA_ERR_*); the message of the last failure on a context is read with
 * har_cuda_last_error.  No function aborts, panics or falls back to the CPU:
 * a missing device or kernel is reported as an error status (fail-closed,
 * as har/crates/har-serve/src/vulkan.rs:18-19 requires of a GPU backend).
 *
 * Threading: one context owns one CUDA stream; a context is not
 * thread-safe (like the reference's &self/RefCell models, moe.rs:47-53) and
 * must be externally locked if shared.  Device pointers passed in ("_dev")
 * must belong to the context's device; host pointers ("_host") are
 * caller-owned and are copied in/out within the call.
 *
 * Layouts (identical to GGUF, so `*_exps` tensors upload unchanged):
 *   Q4_K tensor:  [E][N][K/256] super-blocks of 144 B (f16 d @0, f16 dmin @2,
 *                 12 B 6-bit scales/mins @4, 128 B nibbles @16),
 *                 expert e at byte e*N*(K/256)*144
 *                 (har/crates/har-demo/src/bin/har-native-qwen35moe.rs:664-667).
 *   Q8_K row:     [K/256] blocks of 292 B (f32 d @0, int8 qs[256] @4,
 *                 int16 bsums[16] @260).
 *   activations:  f32 row-major [M][K]; outputs f32 row-major [M][N].
 */
#ifndef HAR_CUDA_H
#define HAR_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HAR_CUDA_ABI_VERSION 1

/* status codes */
#define HAR_CUDA_OK 0
#define HAR_CUDA_ERR_ARG (-1)         /* null pointer / bad enum / bad size */
#define HAR_CUDA_ERR_GEOMETRY (-2)    /* shape mismatch (K not a multiple of 256, ...) */
#define HAR_CUDA_ERR_CUDA (-3)        /* a CUDA runtime call failed */
#define HAR_CUDA_ERR_NCCL (-4)        /* an NCCL call failed */
#define HAR_CUDA_ERR_TIMEOUT (-5)     /* a bounded wait expired (host or device) */
#define HAR_CUDA_ERR_NOT_INIT (-6)    /* context / handle not initialised */
#define HAR_CUDA_ERR_OOM (-7)         /* device allocation failed */
#define HAR_CUDA_ERR_UNSUPPORTED (-8) /* shape/mode this build does not implement */
#define HAR_CUDA_ERR_DEVICE (-9)      /* a kernel reported an error word */

/* activation kinds for har_cuda_q4k_gemv */
#define HAR_CUDA_ACT_F32 0 /* x is f32 [M][K]: HAR's f32-activation arithmetic */
#define HAR_CUDA_ACT_Q8K 1 /* x is Q8_K [M][K/256][292 B]: integer dot products */

/* flags for har_cuda_moe_ffn */
#define HAR_CUDA_MOE_ADD_RESIDUAL 0x1u /* y = x + moe(x), as execute_layer_cpu */
#define HAR_CUDA_MOE_ACT_Q8K 0x2u      /* quantise activations to Q8_K: every expert on the
                                          CUDA-core GEMVs (integer dots); not with FORCE_TC */
#define HAR_CUDA_MOE_FORCE_GEMV 0x4u   /* every expert on the CUDA-core GEMV path */
#define HAR_CUDA_MOE_FORCE_TC 0x8u     /* every expert on the tcgen05 tensor-core path */
#define HAR_CUDA_MOE_EMPTY_SLOTS 0x10u /* expert id -1 marks an empty slot (no contribution);
                                          used by the expert-parallel exchange */
#define HAR_CUDA_MOE_TC_F16W 0x20u     /* tensor-core experts round each dequantised weight
                                          to f16 (faster; max relative error ~4e-4, not
                                          HAR's 5e-5 RMS verdict, which the default meets) */
#define HAR_CUDA_MOE_DECODE 0x40u      /* decode path for T <= 8 tokens: two launches per
                                          layer, no grouping, f32 on CUDA cores (HAR's
                                          verdict met); larger T returns GEOMETRY */

typedef struct har_cuda_ctx har_cuda_ctx;
typedef struct har_cuda_weights har_cuda_weights;
typedef struct har_cuda_moe_layer har_cuda_moe_layer;
typedef struct har_cuda_ep har_cuda_ep;
typedef struct har_cuda_gguf har_cuda_gguf;

/* ---- context ------------------------------------------------------------
 * Replaces the device/queue pair HAR opens per model
 * (har/crates/har-vulkan/src/lib.rs:236 Device::open, :1673 Queue::submit_compute). */
int32_t har_cuda_abi_version(void);
int32_t har_cuda_ctx_create(int32_t device, har_cuda_ctx **out);
int32_t har_cuda_ctx_destroy(har_cuda_ctx *ctx);
/* Copies the last error message (NUL-terminated, truncated to len). */
int32_t har_cuda_last_error(const har_cuda_ctx *ctx, char *buf, size_t len);
/* Launch on a caller-owned cudaStream_t (NULL restores the context's own,
 * a non-blocking stream; pass cudaStreamLegacy, 0x1, to run on the legacy
 * default stream and order with other default-stream work). */
int32_t har_cuda_ctx_set_stream(har_cuda_ctx *ctx, void *cuda_stream);
/* Experts with at least `min_tokens` tokens in a moe_ffn call run on the
 * tensor-core (tcgen05) kernels, the rest on the CUDA-core GEMV kernels;
 * 0 restores the default (1: every expert, when the layer's shapes allow).
 * A tuning knob of this library; the reference has no counterpart. */
int32_t har_cuda_ctx_set_tc_min_tokens(har_cuda_ctx *ctx, int32_t min_tokens);
/* Bounded wait for the context's stream (replaces the unbounded
 * TimelineEvent::wait, har/crates/har-vulkan/src/lib.rs:2168-2175). Also
 * checks the device error word written by kernels with bounded waits. */
int32_t har_cuda_synchronize(har_cuda_ctx *ctx, int64_t timeout_ms);
/* Number of kernels this context has launched (instrumentation). */
int64_t har_cuda_launch_count(const har_cuda_ctx *ctx);

/* ---- weights ------------------------------------------------------------
 * Replaces the staging->device-local copy in VulkanQ4KModel::open /
 * VulkanBatchedModel::open (har/crates/har-serve/src/vulkan.rs:49-119,303-386). */
int32_t har_cuda_weights_upload_q4k(har_cuda_ctx *ctx, const void *host_bytes, int64_t E,
                                    int64_t N, int64_t K, har_cuda_weights **out);
/* Borrow an existing 16-byte-aligned device buffer (not freed by the library). */
int32_t har_cuda_weights_wrap_q4k(har_cuda_ctx *ctx, const void *dev_bytes, int64_t E,
                                  int64_t N, int64_t K, har_cuda_weights **out);
/* Any supported GGML block type: the type ids HAR's GGUF reader matches
 * (har/crates/har-demo/src/bin/har-native-qwen35moe.rs:37-41), rows of
 * K/256 super-blocks (Q4_K 144 B, Q6_K 210 B; row_bytes_for_type, :176-199;
 * Q3_K 110 B, har/crates/har-model/src/lib.rs:591), laid out [E][N][K/256]
 * like the GGUF expert tensors.  Each entry point accepts only the type it
 * computes on (HAR_CUDA_ERR_UNSUPPORTED otherwise): Q4_K for the Q4_K GEMV and
 * the MoE layers, Q6_K for har_cuda_q6k_gemv, Q3_K for har_cuda_q3k_gemv. */
#define HAR_CUDA_GGML_F32 0
#define HAR_CUDA_GGML_Q3_K 11
#define HAR_CUDA_GGML_Q4_K 12
#define HAR_CUDA_GGML_Q6_K 14
int32_t har_cuda_weights_upload(har_cuda_ctx *ctx, int32_t ggml_type, const void *host_bytes,
                                int64_t E, int64_t N, int64_t K, har_cuda_weights **out);
int32_t har_cuda_weights_wrap(har_cuda_ctx *ctx, int32_t ggml_type, const void *dev_bytes,
                              int64_t E, int64_t N, int64_t K, har_cuda_weights **out);
int32_t har_cuda_weights_free(har_cuda_weights *w);
const void *har_cuda_weights_device_ptr(const har_cuda_weights *w);

/* ---- Q8_K activation quantisation ---------------------------------------
 * No reference counterpart (the reference only names q8_k_matvec,
 * har/crates/har-lang-compiler/src/idea_registry.rs:122, and records the
 * 292 B geometry, benchmarks/local-bench/crates/lb-model/src/lib.rs:88).
 * x_dev f32 [M][K] -> out_dev [M][K/256][292 B]. */
int32_t har_cuda_q8k_quantize(har_cuda_ctx *ctx, const float *x_dev, int64_t M, int64_t K,
                              void *out_dev);

/* ---- Q4_K GEMV ------------------------------------------------------------
 * y[m][n] = sum_k W_e[n][k] * x[m][k] for m < M.  Replaces Q4KModel::matvec
 * (har/crates/har-serve/src/q4k.rs:170-188), expert_matvec
 * (har/crates/har-demo/src/bin/har-native-qwen35moe.rs:626-689) and the
 * q4k_gemv / q4k_batched_gemv dispatches (har/crates/har-serve/src/vulkan.rs:131-191,402-462).
 * act_kind HAR_CUDA_ACT_F32: x_dev is f32 [M][K]; HAR_CUDA_ACT_Q8K: Q8_K rows. */
int32_t har_cuda_q4k_gemv(har_cuda_ctx *ctx, const har_cuda_weights *w, int64_t expert,
                          const void *x_dev, int32_t act_kind, int64_t M, float *y_dev);

/* ---- Q6_K GEMV --------------------------------------------------------------
 * y[m][n] = sum_k W_e[n][k] * x[m][k] for Q6_K weights (ql[128], qh[64], int8
 * scales[16], f16 d per 210-byte super-block) and f32 activations x_dev
 * [M][K] (16-byte aligned); y_dev f32 [M][N].  Replaces the Q6_K arm of
 * dot_quant_row / q6k_dot (har/crates/har-demo/src/bin/har-native-qwen3.rs:174-232)
 * as NativeQwen35Moe::matvec reaches it for Q6_K tensors
 * (har/crates/har-demo/src/bin/har-native-qwen35moe.rs:551-556,583-624). */
int32_t har_cuda_q6k_gemv(har_cuda_ctx *ctx, const har_cuda_weights *w, int64_t expert,
                          const float *x_dev, int64_t M, float *y_dev);

/* ---- Q3_K GEMV --------------------------------------------------------------
 * y[m][n] = sum_k W_e[n][k] * x[m][k] for Q3_K weights and f32 activations
 * x_dev [M][K] (16-byte aligned); y_dev f32 [M][N].  The reference records
 * Q3_K's geometry only (GGML type 11, 110 B per 256 values,
 * har/crates/har-model/src/lib.rs:591) and no arithmetic; the block layout is
 * GGUF's: hmask[32] (high bits), qs[64] (2-bit planes), 12 bytes of packed
 * 6-bit sub-block scales (offset 32), f16 d. */
int32_t har_cuda_q3k_gemv(har_cuda_ctx *ctx, const har_cuda_weights *w, int64_t expert,
                          const float *x_dev, int64_t M, float *y_dev);

/* ---- router top-k ---------------------------------------------------------
 * Per token: softmax over all E logits with max subtraction, experts ordered
 * by probability descending then lower index, first k taken, weights
 * renormalised by their sum (both sums clamped to >= 1e-9).  Bit-exact with
 * routed_moe (har/crates/har-demo/src/bin/har-native-qwen35moe.rs:1167-1204).
 * logits_dev f32 [T][E]; ids_dev int32 [T][k]; weights_dev f32 [T][k]. */
int32_t har_cuda_route_topk(har_cuda_ctx *ctx, const float *logits_dev, int64_t T, int32_t E,
                            int32_t k, int32_t *ids_dev, float *weights_dev);

/* ---- router GEMV ------------------------------------------------------------
 * logits[t][e] = sum_h gate_inp[e][h] * x[t][h] for the f32 router matrix
 * ffn_gate_inp [E][H]: one f32 accumulator per (token, expert), h ascending,
 * each product rounded before it is added — bit-exact with routed_moe's
 * self.matvec(ffn_gate_inp) (har/crates/har-demo/src/bin/har-native-qwen35moe.rs:1168-1172),
 * whose F32 row dot is dot_f32_row (:154-163).
 * gate_inp_dev f32 [E][H]; x_dev f32 [T][H]; logits_dev f32 [T][E]. */
int32_t har_cuda_router_logits(har_cuda_ctx *ctx, const float *gate_inp_dev, int32_t E,
                               int64_t H, const float *x_dev, int64_t T, float *logits_dev);
/* routed_moe's whole selection on the device: the router GEMV above, then
 * har_cuda_route_topk's softmax + top-k (har-native-qwen35moe.rs:1167-1204).
 * The logits live in the context's scratch arena.  ids_dev int32 [T][k],
 * weights_dev f32 [T][k] (the RouteRecord's experts and weights). */
int32_t har_cuda_route(har_cuda_ctx *ctx, const float *gate_inp_dev, int32_t E, int64_t H,
                       const float *x_dev, int64_t T, int32_t k, int32_t *ids_dev,
                       float *weights_dev);

/* ---- expert-major grouping -------------------------------------------------
 * groups[e] = entries (t*k + slot) routed to e, in position order
 * (har/crates/har-serve/src/moe.rs:195-202).  counts_dev int32 [E],
 * offsets_dev int32 [E+1], order_dev int32 [T*k]. */
int32_t har_cuda_group_by_expert(har_cuda_ctx *ctx, const int32_t *ids_dev, int64_t T,
                                 int32_t k, int32_t E, int32_t *counts_dev,
                                 int32_t *offsets_dev, int32_t *order_dev);

/* ---- MoE FFN layer --------------------------------------------------------
 * A layer = gate/up [E][I][H/256], down [E][H][I/256] Q4_K tensors plus an
 * optional shared expert (three 1-expert tensors of the same shapes) and an
 * optional f32 [H] shared-expert gate row (NULL: gate weight 1.0).
 * Mirrors the tensor set compose_moe_route reads per layer
 * (har/crates/har-demo/src/bin/har-native-qwen35moe.rs:979-1048). */
int32_t har_cuda_moe_layer_create(har_cuda_ctx *ctx, const har_cuda_weights *gate,
                                  const har_cuda_weights *up, const har_cuda_weights *down,
                                  const har_cuda_weights *sh_gate,
                                  const har_cuda_weights *sh_up,
                                  const har_cuda_weights *sh_down,
                                  const float *sh_gate_inp_dev, har_cuda_moe_layer **out);
int32_t har_cuda_moe_layer_free(har_cuda_moe_layer *layer);

/* y[t] = sum_s weights[t][s] * down_e(silu(gate_e x_t) * up_e x_t)
 *        + sigmoid(sh_gate_inp . x_t) * shared(x_t)   [+ x_t with ADD_RESIDUAL],
 * experts e = ids[t][s] in slot order; device pointers.  Replaces
 * compose_moe_route / routed_moe's expert loop and MoEModel::forward_batch's
 * expert-major grouping (har/crates/har-serve/src/moe.rs:182-255). */
int32_t har_cuda_moe_ffn(har_cuda_ctx *ctx, const har_cuda_moe_layer *layer,
                         const float *x_dev, int64_t T, int32_t k, const int32_t *ids_dev,
                         const float *weights_dev, float *y_dev, uint32_t flags);
/* routed_moe (har/crates/har-demo/src/bin/har-native-qwen35moe.rs:1167-1215)
 * on the device: har_cuda_route with the layer's E and H (gate_inp_dev f32
 * [E][H], the layer's ffn_gate_inp; NULL = the router a layer loaded from
 * GGUF carries), writing the route record to ids_dev
 * [T][k] / weights_dev [T][k], then har_cuda_moe_ffn on that routing. */
int32_t har_cuda_routed_moe(har_cuda_ctx *ctx, const har_cuda_moe_layer *layer,
                            const float *gate_inp_dev, const float *x_dev, int64_t T, int32_t k,
                            int32_t *ids_dev, float *weights_dev, float *y_dev, uint32_t flags);
/* A stack of L routed layers in one call: for each layer, routed_moe's
 * selection on the device from that layer's input (gate_inp_devs[l], or the
 * layer's own GGUF router when gate_inp_devs or its entry is NULL), then the
 * layer, y_l = moe_l(y_{l-1}) [+ residual with HAR_CUDA_MOE_ADD_RESIDUAL] —
 * the FFN half of NativeQwen35Moe::forward's layer loop
 * (har/crates/har-demo/src/bin/har-native-qwen35moe.rs:1152-1215), attention
 * and norms omitted.  Route records go to ids_dev / weights_dev [L][T][k];
 * x_dev and y_dev may alias.  All work is enqueued on the context's stream. */
int32_t har_cuda_routed_moe_stack(har_cuda_ctx *ctx, const har_cuda_moe_layer *const *layers,
                                  int32_t L, const float *const *gate_inp_devs,
                                  const float *x_dev, int64_t T, int32_t k, int32_t *ids_dev,
                                  float *weights_dev, float *y_dev, uint32_t flags);
/* The same with host buffers: copies x/ids/weights in and y out on the
 * context's stream and waits (bounded) — the call a BatchStepModel makes. */
int32_t har_cuda_moe_ffn_host(har_cuda_ctx *ctx, const har_cuda_moe_layer *layer,
                              const float *x_host, int64_t T, int32_t k,
                              const int32_t *ids_host, const float *weights_host,
                              float *y_host, uint32_t flags);
/* har_cuda_moe_ffn without any device allocation.  No counterpart in the
 * reference: it exists for callers that cannot call cudaMalloc — runtimes that
 * reserve the GPU's memory up front for their own pools, and hot loops that
 * cannot take the synchronisation an allocation may imply.  Scratch comes from
 * a static device array of HAR_CUDA_NOALLOC_SCRATCH_BYTES held by every GPU
 * that loads the library until exit; calls needing more return
 * HAR_CUDA_ERR_GEOMETRY (T <= 144 tokens at E = 512, H = 2048, I = 512, k = 10
 * with f32 activations, 276 with HAR_CUDA_MOE_ACT_Q8K).
 * The first call in each CUDA context looks up the array's address in that
 * context (make it before any stream capture); the address is cached per
 * context, so a device reset or a non-primary context gets its own lookup.  All calls on a device share the array: calls that overlap
 * on the GPU race and must be serialised by the caller.  Arguments, results
 * and error behaviour are those of har_cuda_moe_ffn. */
#define HAR_CUDA_NOALLOC_SCRATCH_BYTES (32u << 20)
int32_t har_cuda_moe_ffn_noalloc(har_cuda_ctx *ctx, const har_cuda_moe_layer *layer,
                                 const float *x_dev, int64_t T, int32_t k,
                                 const int32_t *ids_dev, const float *weights_dev, float *y_dev,
                                 uint32_t flags);
/* A stack of L layers applied in order (y_l = moe_l(y_{l-1}) [+ residual]),
 * ids/weights [L][T][k]; x_dev and y_dev may alias.  Attention and norms
 * between layers are outside this path. */
int32_t har_cuda_moe_stack(har_cuda_ctx *ctx, const har_cuda_moe_layer *const *layers,
                           int32_t L, const float *x_dev, int64_t T, int32_t k,
                           const int32_t *ids_dev, const float *weights_dev, float *y_dev,
                           uint32_t flags);

/* The stack with host buffers (x [T][H], ids/weights [L][T][k], y [T][H]):
 * copies in, runs, copies out and waits (bounded).  A call repeated with the
 * same layers, shapes, flags and stream replays a CUDA graph of its device work
 * (captured on the second such call; not on the legacy or per-thread default
 * stream, where capture is not allowed); the inputs are read afresh every call.
 * Layers are identified by an id assigned at creation, never by address, so a
 * layer freed and recreated at the same address is a new key. */
int32_t har_cuda_moe_stack_host(har_cuda_ctx *ctx, const har_cuda_moe_layer *const *layers,
                                int32_t L, const float *x_host, int64_t T, int32_t k,
                                const int32_t *ids_host, const float *weights_host,
                                float *y_host, uint32_t flags);

/* ---- GGUF expert loader ------------------------------------------------------
 * Opens a GGUF file (versions 1-3) and reads its directory the way
 * GgufReader::inspect does (har/crates/har-model/src/lib.rs:126-399):
 * metadata (general.alignment, default 32), tensor infos, the aligned data
 * offset and each tensor's payload size from the GGML type tables
 * (:605-640).  Host-only: no GPU is needed to open or query a file.  On
 * failure the message goes to err (may be NULL).  The handle keeps the file
 * open and, once a tensor has been loaded, two 64 MiB pinned staging buffers;
 * it is not thread-safe. */
int32_t har_cuda_gguf_open(const char *path, char *err, size_t err_len, har_cuda_gguf **out);
int32_t har_cuda_gguf_close(har_cuda_gguf *g);
int32_t har_cuda_gguf_last_error(const har_cuda_gguf *g, char *buf, size_t len);
int32_t har_cuda_gguf_header(const har_cuda_gguf *g, uint32_t *version, uint64_t *tensor_count,
                             uint64_t *metadata_count, uint64_t *alignment,
                             uint64_t *data_offset);
/* Tensor `index` (file order): name, GGML type, rank, dims (up to 16, GGML
 * order: dims[0] is the row length), absolute file offset, payload bytes. */
int32_t har_cuda_gguf_tensor_info(const har_cuda_gguf *g, int64_t index, char *name,
                                  size_t name_len, uint32_t *ggml_type, uint32_t *rank,
                                  uint64_t *dims, uint64_t *file_offset, uint64_t *payload_bytes);
/* Index of the tensor called `name`, or -1. */
int64_t har_cuda_gguf_find(const har_cuda_gguf *g, const char *name);
/* A metadata value as a number, as metadata_number reads it
 * (har/crates/har-model/src/lib.rs:541-543), or a string value. */
int32_t har_cuda_gguf_meta_u64(const har_cuda_gguf *g, const char *key, uint64_t *value);
int32_t har_cuda_gguf_meta_string(const har_cuda_gguf *g, const char *key, char *buf,
                                  size_t len);
/* Upload a Q4_K or Q6_K tensor straight into the device layout: GGML dims
 * [K, N, E] (an `*_exps` tensor, expert e at e*N*row_bytes as expert_matvec
 * reads it, har/crates/har-demo/src/bin/har-native-qwen35moe.rs:626-689, and
 * as ExpertIndex slices it, har/crates/har-storage/src/gguf.rs:300-403) or
 * [K, N] (E = 1), byte for byte.  The weights own their device memory. */
int32_t har_cuda_weights_from_gguf(har_cuda_ctx *ctx, har_cuda_gguf *g, const char *name,
                                   har_cuda_weights **out);
/* Copy an F32 tensor of exactly `count` elements to dst_dev. */
int32_t har_cuda_gguf_read_f32(har_cuda_ctx *ctx, har_cuda_gguf *g, const char *name,
                               float *dst_dev, int64_t count);
/* One MoE layer from blk.<layer>.ffn_{gate,up,down}_exps.weight, the shared
 * expert ffn_{gate,up,down}_shexp.weight and its gate row
 * ffn_gate_inp_shexp.weight when present, and the f32 router
 * ffn_gate_inp.weight when present — the tensors routed_moe and
 * compose_moe_route read (har-native-qwen35moe.rs:979-1048,1167-1215).  The
 * layer owns all of them (har_cuda_moe_layer_free releases them);
 * har_cuda_routed_moe with gate_inp_dev = NULL uses the layer's router. */
int32_t har_cuda_moe_layer_from_gguf(har_cuda_ctx *ctx, har_cuda_gguf *g, int32_t layer,
                                     har_cuda_moe_layer **out);

/* ---- expert parallelism over the GPUs of one box (NVLink peer memory, NCCL) --------------
 * No counterpart in the reference, which runs every expert on one CPU
 * (compose_moe_route, har-native-qwen35moe.rs:979-1048): this is the router-to-
 * expert dispatch of a sharded deployment.  Rank r of G holds the routed experts
 * [r*E/G, (r+1)*E/G) of every layer as a `local` layer (no shared expert) and the
 * shared expert as a one-expert `shared` layer (replicated on every rank), plus
 * the shared expert's gate row.  Per layer: token rows go to the ranks holding
 * their experts, each rank runs its experts, partial sums come back, and the
 * tokens' rank adds residual, shared expert and partial sums.  Results equal
 * har_cuda_moe_ffn on the unsharded layer up to f32 summation order.  All
 * ranks call collectively with the same T, k and flags (ADD_RESIDUAL,
 * ACT_Q8K, FORCE_*).
 * By default the rows move in two grouped NCCL send/recv rounds.  With
 * har_cuda_ep_set_p2p(ep, 1) they move through peer memory instead: every
 * rank's exchange window is mapped into the other ranks by CUDA IPC on the
 * first call (collective;
 * again when a call needs a larger window, and that call must not be under
 * graph capture), and each rank pulls over NVLink the token rows that have an
 * expert of its own and the partial sums of its own tokens, synchronised by
 * epoch flags whose waits give up after the communicator's timeout (the next
 * har_cuda_synchronize then returns HAR_CUDA_ERR_TIMEOUT, and the
 * communicator should be aborted).
 * When any rank cannot map every window (ranks sharing a GPU, no peer access)
 * all ranks keep the NCCL rounds. */
/* The two device steps of the exchange on their own, without a communicator:
 * for callers that move the rows with their own transport, and for checking
 * the plan and the combine on one GPU.
 * har_cuda_ep_plan writes, for every destination d < world and token t < T,
 * row d*T + t: sids [world*T][k] = the d-local expert id of each slot (-1 where
 * the expert lives on another rank; rank d holds experts [d*E/world,
 * (d+1)*E/world)), sw [world*T][k] = the slot's weight (0 where -1), and
 * sx [world*T][H] = x[t] when at least one slot lives on d (the row is left
 * unwritten otherwise).  Out-of-range ids set the device error word
 * (HAR_CUDA_ERR_DEVICE at the next har_cuda_synchronize).
 * har_cuda_ep_combine writes y[t] = (x[t] with HAR_CUDA_MOE_ADD_RESIDUAL) +
 * shared[t] + back[0][t] + ... + back[world-1][t], each addition rounded to
 * f32 in that order; shared_dev may be null (no shared expert) and x_dev may
 * alias y_dev. */
int32_t har_cuda_ep_plan(har_cuda_ctx *ctx, const float *x_dev, int64_t H, int64_t T, int32_t k,
                         const int32_t *ids_dev, const float *weights_dev, int32_t E, int32_t world,
                         float *sx_dev, int32_t *sids_dev, float *sw_dev);
int32_t har_cuda_ep_combine(har_cuda_ctx *ctx, const float *x_dev, int64_t H, int64_t T,
                            int32_t world, const float *shared_dev, const float *back_dev,
                            uint32_t flags, float *y_dev);
/* An NCCL unique id (rank 0 creates it; the caller broadcasts the bytes). */
int32_t har_cuda_ep_unique_id(uint8_t *out, size_t len);
/* Collective: every rank of `world` joins the communicator on ctx's device.
 * The communicator is non-blocking and every wait on it is bounded (this call
 * waits up to 300 s for all ranks to join; each exchange's enqueue up to the
 * same bound): on expiry the communicator is aborted and the call returns
 * HAR_CUDA_ERR_TIMEOUT, replacing the unbounded device-fence waits of the
 * reference's device layer (har-vulkan/src/lib.rs:2174) with the fail-closed
 * rule of its serving seam (har-serve/src/vulkan.rs:18-19). */
int32_t har_cuda_ep_create(har_cuda_ctx *ctx, const uint8_t *unique_id, size_t len, int32_t world,
                           int32_t rank, har_cuda_ep **out);
/* The same with the bound given: timeout_ms for joining and for each exchange. */
int32_t har_cuda_ep_create_timeout(har_cuda_ctx *ctx, const uint8_t *unique_id, size_t len,
                                   int32_t world, int32_t rank, int64_t timeout_ms,
                                   har_cuda_ep **out);
/* Abort the communicator: its NCCL work in flight ends with an error instead of
 * waiting for peers (call it when har_cuda_synchronize timed out on an exchange
 * whose peer is gone); later EP calls on it return HAR_CUDA_ERR_NOT_INIT.  The
 * handle still needs har_cuda_ep_free. */
int32_t har_cuda_ep_abort(har_cuda_ep *ep);
/* Collective when windows were mapped (every rank calls it): unmaps the peers'
 * windows, then frees this rank's after a barrier over the communicator
 * (without one — aborted, or a rank gone — the window stays allocated). */
int32_t har_cuda_ep_free(har_cuda_ep *ep);
/* Choose the transport of later calls: on != 0 peer memory where every rank
 * can map every window, 0 the NCCL rounds (the default).  Call it with the
 * same value on every rank. */
int32_t har_cuda_ep_set_p2p(har_cuda_ep *ep, int32_t on);
/* The transport of the last call: 1 peer memory, 0 NCCL (chosen, or not yet
 * set up), -1 NCCL because some rank could not map the windows. */
int32_t har_cuda_ep_exchange_mode(const har_cuda_ep *ep);
/* One layer; ids are global expert ids [T][k] of this rank's T tokens. */
int32_t har_cuda_ep_moe_ffn(har_cuda_ctx *ctx, har_cuda_ep *ep, const har_cuda_moe_layer *local,
                            const har_cuda_moe_layer *shared, const float *gate_inp_dev,
                            const float *x_dev, int64_t T, int32_t k, const int32_t *ids_dev,
                            const float *weights_dev, float *y_dev, uint32_t flags);
/* L layers in order (ids/weights [L][T][k]); shared_layers and gate_inp_devs may
 * be null; x_dev and y_dev may alias. */
int32_t har_cuda_ep_moe_stack(har_cuda_ctx *ctx, har_cuda_ep *ep,
                              const har_cuda_moe_layer *const *local_layers,
                              const har_cuda_moe_layer *const *shared_layers,
                              const float *const *gate_inp_devs, int32_t L, const float *x_dev,
                              int64_t T, int32_t k, const int32_t *ids_dev,
                              const float *weights_dev, float *y_dev, uint32_t flags);

/* ---- expert-slot residency (ExpertSlotTable, har/crates/har-vulkan/src/lib.rs:1233-1460) ---
 * A bounded table of device slots, each holding one projection of one expert,
 * for deployments whose experts do not all stay resident.  The rules are the
 * reference's: a slot is Free, Uploading (reserve), Ready (mark_ready once the
 * upload's event completed), InFlight (acquire_for_dispatch) and Ready again
 * (release once the dispatch's event completed), or Free (evict, never while in
 * flight); every transition takes the next value of a monotone epoch (the
 * caller's LRU order, read back with snapshot).  Events are cudaEvent_t handles
 * passed as void*, complete when cudaEventQuery reports so; an incomplete
 * event is HAR_CUDA_ERR_ARG with the reference's message.  A table created
 * with ctx == NULL has no storage (the state machine alone) and takes only
 * NULL events, meaning "already complete".  To serve a MoE layer from slots,
 * create one table per projection, keep an expert's three projections at the
 * same slot index (identical operation sequences give identical indices), wrap
 * each table's storage with har_cuda_weights_wrap_q4k(ctx, storage, count, N, K)
 * and pass slot ids as the expert ids. */
typedef struct har_cuda_slot_table har_cuda_slot_table;
#define HAR_CUDA_PROJ_GATE 0u
#define HAR_CUDA_PROJ_UP 1u
#define HAR_CUDA_PROJ_DOWN 2u
#define HAR_CUDA_SLOT_FREE 0
#define HAR_CUDA_SLOT_UPLOADING 1
#define HAR_CUDA_SLOT_READY 2
#define HAR_CUDA_SLOT_IN_FLIGHT 3
typedef struct {          /* ExpertSlotKey (lib.rs:1239-1244) */
  uint32_t layer, expert_id, projection;  /* projection: HAR_CUDA_PROJ_* */
  uint64_t generation;    /* 0 is reserved */
} har_cuda_slot_key;
typedef struct {          /* ExpertSlotSnapshot (lib.rs:1253-1260) */
  uint32_t slot_id;
  har_cuda_slot_key key;
  int32_t state;          /* HAR_CUDA_SLOT_* */
  uint64_t upload_epoch, last_use_epoch;
  int32_t ready;
} har_cuda_slot_snapshot;
/* create_expert_slot_table (lib.rs:925-970): count x slot_bytes of device
 * storage (none when ctx is NULL), every slot Free, epochs from 1. */
int32_t har_cuda_slot_table_create(har_cuda_ctx *ctx, uint32_t slot_count, uint64_t slot_bytes,
                                   har_cuda_slot_table **out);
/* Waits for the context's stream, then frees the storage. */
int32_t har_cuda_slot_table_free(har_cuda_slot_table *table);
int32_t har_cuda_slot_table_storage(har_cuda_slot_table *table, void **dev, uint64_t *bytes);
int32_t har_cuda_slot_table_last_error(const har_cuda_slot_table *table, char *buf, size_t len);
/* reserve (lib.rs:1282-1314): the first Free slot takes the key. */
int32_t har_cuda_slot_reserve(har_cuda_slot_table *table, const har_cuda_slot_key *key,
                              uint32_t *slot_id);
/* mark_upload_submitted (lib.rs:1315-1333), for a caller that moved the bytes. */
int32_t har_cuda_slot_mark_upload_submitted(har_cuda_slot_table *table, uint32_t slot_id,
                                            void *cuda_event);
/* Copies bytes (<= slot_bytes) from host memory into the slot on the context's
 * stream and records the table's event for it: mark_upload_submitted for the
 * library's own upload. */
int32_t har_cuda_slot_upload(har_cuda_slot_table *table, uint32_t slot_id, const void *host_src,
                             uint64_t bytes);
/* mark_ready (lib.rs:1334-1368); cuda_event NULL = the submitted upload's. */
int32_t har_cuda_slot_mark_ready(har_cuda_slot_table *table, uint32_t slot_id, void *cuda_event);
/* acquire_for_dispatch (lib.rs:1369-1394): Ready -> InFlight, the slot's record. */
int32_t har_cuda_slot_acquire(har_cuda_slot_table *table, const har_cuda_slot_key *key,
                              har_cuda_slot_snapshot *out);
/* release_from_dispatch (lib.rs:1395-1419) */
int32_t har_cuda_slot_release(har_cuda_slot_table *table, uint32_t slot_id, void *cuda_event);
/* evict (lib.rs:1420-1450) */
int32_t har_cuda_slot_evict(har_cuda_slot_table *table, uint32_t slot_id, void *cuda_event);
/* snapshot (lib.rs:1451-1456): writes min(cap, count) records, *n = count. */
int32_t har_cuda_slot_table_snapshot(har_cuda_slot_table *table, har_cuda_slot_snapshot *out,
                                     uint32_t cap, uint32_t *n);

/* ---- profiling (the role of TimestampQuery, har/crates/har-vulkan/src/lib.rs:2221-2257) ---
 * Between begin and end every kernel the context launches is bracketed by
 * CUDA events on its stream; end waits for the stream and returns up to cap
 * (kernel name, milliseconds) records: names '\n'-separated in `names`. */
int32_t har_cuda_profile_begin(har_cuda_ctx *ctx);
int32_t har_cuda_profile_end(har_cuda_ctx *ctx, char *names, size_t names_len, float *ms,
                             int64_t cap, int64_t *count);

/* ---- synthetic inputs (bench/test generator, not a reference function) ---
 * Fills dev_bytes with rows x K N(mean,std) values quantised to Q4_K by the
 * same quantiser as the oracle's haro_q4k_quantize_row, element (r, c) being
 * normal index (row0 + r)*K + c of `seed`. */
int32_t har_cuda_gen_q4k(har_cuda_ctx *ctx, void *dev_bytes, int64_t rows, int64_t K,
                         uint64_t seed, int64_t row0, float mean, float std);

#ifdef __cplusplus
}
#endif
#endif
