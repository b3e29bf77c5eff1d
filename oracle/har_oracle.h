/*
 * har_oracle.h — CPU restatement of HAR's Q4_K MoE-FFN path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA path:
 * only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
 * load it.  The product (libhar_cuda.so) never links or calls it.
 *
 * The reference (leoinfer/remora-lab, HAR) is Rust; no Rust toolchain exists
 * in this build image, so each function below restates the cited Rust
 * function in C with the same f32 operation order.  Build flags
 * (-O2 -ffp-contract=off, no -ffast-math) keep IEEE single-precision
 * semantics identical to Rust's (Rust never contracts or reassociates f32).
 * exp() comes from glibc's expf, the libm that Rust's f32::exp links on Linux.
 *
 * Pinning: the reference's known-answer tests for this path (f16 values,
 * zero blocks, the 256.0 Vulkan smoke value, top-k tie order, Q4_K row
 * geometry) are committed as tests/golden/reference_kats.json and checked in
 * tests/test_oracle_kats.py.  No reference test pins full GEMV outputs, the
 * Q8_K quantiser or the Q4_K quantiser: those two quantisers are this
 * project's own (the formats belong to ggml, which the reference neither
 * vendors nor depends on), so their parity is unpinned.
 */
#ifndef HAR_ORACLE_H
#define HAR_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HARO_QK_K 256
#define HARO_Q4K_BLOCK_BYTES 144
#define HARO_Q8K_BLOCK_BYTES 292
#define HARO_Q6K_BLOCK_BYTES 210
#define HARO_Q3K_BLOCK_BYTES 110
#define HARO_ROUTER_EPS 1.0e-9f

/* ---- a1: binary16 -> f32 ------------------------------------------------ */
/* har/crates/har-serve/src/q4k.rs:22-50 (arithmetic construction). */
float haro_f16_to_f32(uint8_t b0, uint8_t b1);
/* har/crates/har-demo/src/bin/har-native-qwen3.rs:116-136 (bit construction). */
float haro_half_to_f32(uint16_t v);
/* f32 -> binary16, round to nearest even (this project's quantiser helper). */
uint16_t haro_f32_to_f16_rne(float f);

/* ---- a2: 6-bit scale/min unpack ----------------------------------------- */
/* har/crates/har-serve/src/q4k.rs:60-74 */
uint32_t haro_scale_at(const uint8_t *block, int index);
uint32_t haro_min_at(const uint8_t *block, int index);
/* har/crates/har-demo/src/bin/har-native-qwen3.rs:138-147 (scales = block+4) */
void haro_scale_min(const uint8_t *scales, int index, uint8_t *sc, uint8_t *m);

/* ---- a3: dequant --------------------------------------------------------- */
/* har/crates/har-serve/src/q4k.rs:77-89 */
float haro_q4k_dequant(const uint8_t *block, int index);
/* har/crates/har-demo/src/bin/har-native-qwen3.rs:1067-1093 */
void haro_decode_q4k_block(const uint8_t *block, float out[256]);

/* ---- a4: serving-path matvec (config 1's HAR path) ---------------------- */
/* har/crates/har-serve/src/q4k.rs:170-188: one sequential f32 accumulator
 * per row over blocks then the 256 values in index order. */
void haro_q4k_matvec(const uint8_t *w, int64_t rows, int64_t dim,
                     const float *x, float *out);

/* ---- a5: expert-path dot ------------------------------------------------- */
/* har/crates/har-demo/src/bin/har-native-qwen3.rs:149-172 */
float haro_q4k_dot(const uint8_t *block, const float *x);
/* har/crates/har-demo/src/bin/har-native-qwen3.rs:207-232 (Q4_K arm) */
float haro_dot_quant_row(const uint8_t *row, const float *x, int64_t k);
/* ---- Q6_K ------------------------------------------------------------------ */
/* har/crates/har-demo/src/bin/har-native-qwen3.rs:174-205 */
float haro_q6k_dot(const uint8_t *block, const float *x);
/* har/crates/har-demo/src/bin/har-native-qwen3.rs:207-232 (Q6_K arm) */
float haro_dot_quant_row_q6k(const uint8_t *row, const float *x, int64_t k);
/* rows x k Q6_K tensor times x (the per-row dot above for every row) */
void haro_q6k_matvec(const uint8_t *w, int64_t rows, int64_t k, const float *x, float *out);

/* ---- f3: Q3_K (parity unpinned) ------------------------------------------
 * The reference holds only Q3_K's geometry (GGML type 11, 110 bytes per 256
 * values: har/crates/har-model/src/lib.rs:591,
 * benchmarks/local-bench/crates/lb-model/src/lib.rs:84) and no arithmetic;
 * this restates the GGUF block layout as ggml publishes it (block_q3_K and its
 * row dequantisation, ggml's k-quants, the format GGUF files carry): hmask[32]
 * @0, qs[64] @32, 12 bytes of packed 6-bit scales @96, f16 d @108.  Value
 * i = 128n + 32j + l (n < 2, j < 4, l < 32) is
 *   d * (scale[8n + 2j + l/16] - 32) * (((qs[32n + l] >> 2j) & 3) - 4 * !(hmask[l] >> (4n + j) & 1)).
 * No reference vectors exist to pin it: checked against hand-built blocks. */
/* The 6-bit scale of sub-block s (0..15) from the 12 packed bytes. */
int haro_q3k_scale(const uint8_t *scales12, int s);
void haro_q3k_dequant_block(const uint8_t *block, float out[256]);
/* sum over the block of (d * (scale - 32)) * q * x, in index order, in f32. */
float haro_q3k_dot(const uint8_t *block, const float *input);
void haro_q3k_matvec(const uint8_t *w, int64_t rows, int64_t k, const float *x, float *out);
/* har/crates/har-demo/src/bin/har-native-qwen35moe.rs:154-163 */
float haro_dot_f32_row(const float *row, const float *x, int64_t k);

/* har/crates/har-demo/src/bin/har-native-qwen35moe.rs:1168-1172 with :154-163:
 * logits[e] = dot_f32_row(gate_inp[e], x) for the f32 router [E][H]. */
void haro_router_logits(const float *gate_inp, int64_t E, int64_t H, const float *x,
                        float *logits);

/* ---- a6: expert matvec --------------------------------------------------- */
/* har/crates/har-demo/src/bin/har-native-qwen35moe.rs:626-689: tensor of
 * [E][N][K/256] super-blocks, expert e at e*N*row_bytes; rows split into
 * contiguous chunks of ceil(N/workers) over `threads` workers spawned per
 * call (threads <= 0: the host's online CPU count, as available_parallelism). */
void haro_expert_matvec(const uint8_t *tensor, int64_t E, int64_t N, int64_t K,
                        int64_t expert, const float *x, float *y, int threads);

/* ---- a7: SwiGLU expert FFN + weighted combine ---------------------------- */
/* har/crates/har-demo/src/bin/har-native-qwen35moe.rs:203-214 */
float haro_silu(float v);
float haro_sigmoid(float v);
/* har/crates/har-demo/src/bin/har-native-qwen35moe.rs:979-1048, for one token.
 *   w_gate, w_up: [E][I][H/256] Q4_K;  w_down: [E][H][I/256] Q4_K
 *   sh_gate/sh_up/sh_down: the shared expert (one expert of the same shape), or
 *   all NULL for no shared expert; sh_gate_inp: f32[H] shared-expert gate row,
 *   NULL meaning a gate weight of exactly 1.0 (moe.rs:221-233 semantics). */
void haro_compose_moe_route(const uint8_t *w_gate, const uint8_t *w_up,
                            const uint8_t *w_down, const uint8_t *sh_gate,
                            const uint8_t *sh_up, const uint8_t *sh_down,
                            const float *sh_gate_inp, int64_t E, int64_t H,
                            int64_t I, int k, const float *x,
                            const int32_t *experts, const float *weights,
                            float *out, int threads);

/* ---- a8: router softmax + top-k ------------------------------------------ */
/* har/crates/har-demo/src/bin/har-native-qwen35moe.rs:1167-1215 (selection
 * part): softmax over all E with max subtraction, order by probability
 * descending (total_cmp) then lower index, take k, renormalise by the
 * selected sum (both denominators clamped to >= ROUTER_EPS). */
void haro_route_topk(const float *logits, int E, int k, int32_t *ids, float *weights);
/* 0: exp = glibc expf (the reference's f32::exp); 1: correctly rounded exp. */
void haro_set_exp_mode(int mode);
/* glibc's expf restated (Nagy's table-driven method, fused multiply-adds as on
 * x86-64 with FMA), its 2^(i/32) table, and a counter of the floats in a bit
 * pattern range where it differs from the host's expf. */
float haro_expf_restated(float x);
void haro_exp2_table(uint64_t *out);
uint64_t haro_expf_mismatches(uint32_t lo, uint32_t hi, uint32_t *first);

/* ---- a9: expert-major grouping ------------------------------------------- */
/* har/crates/har-serve/src/moe.rs:195-202: groups[e] = positions routed to e
 * in position order.  Output: counts[E], offsets[E+1] (exclusive scan) and
 * order[T*k] = (token*k + slot) entries grouped by expert, stable. */
void haro_group_by_expert(int64_t T, int k, int E, const int32_t *ids,
                          int32_t *counts, int32_t *offsets, int32_t *order);

/* ---- the whole batched layer --------------------------------------------- */
/* compose_moe_route applied per token t (ids/weights [T][k]); when
 * add_residual != 0 the token's input row is added afterwards, as
 * execute_layer_cpu adds ffn_residual (har-native-qwen35moe.rs:1152-1155). */
void haro_moe_ffn(const uint8_t *w_gate, const uint8_t *w_up, const uint8_t *w_down,
                  const uint8_t *sh_gate, const uint8_t *sh_up, const uint8_t *sh_down,
                  const float *sh_gate_inp, int64_t E, int64_t H, int64_t I,
                  int64_t T, int k, const float *x, const int32_t *ids,
                  const float *weights, int add_residual, float *y, int threads);

/* ---- a11: Q8_K activation quantisation (this project's own; unpinned) ---- */
/* 292-byte block: f32 d @0, int8 qs[256] @4, int16 bsums[16] @260.
 *   amax = max|x|; amax == 0 -> d = 0, qs = 0;
 *   else iscale = 127/amax (f32 division), q = clamp(rint(x*iscale), -127, 127),
 *   d = amax/127 (when 127/amax overflows to inf, q = clamp(rint(x/d)) instead);  bsums[g] = sum of qs[16g .. 16g+15]. */
void haro_q8k_quantize(const float *x, int64_t k, uint8_t *out);
/* Q8_K x Q4_K row dot (own design): per super-block, exact int32
 *   I1 = sum_j sc_j * sum_{i in j} q4_i*q8_i,  I2 = sum_j m_j * (bsums[2j]+bsums[2j+1]);
 *   blk = (d_w*d_x)*(float)I1 - (dmin_w*d_x)*(float)I2;  row = sequential sum of blk. */
float haro_q8k_dot_row(const uint8_t *row_q4k, const uint8_t *xq8k, int64_t k);
void haro_q4k_gemv_q8k(const uint8_t *w, int64_t rows, int64_t k,
                       const uint8_t *xq8k, float *out);
/* haro_moe_ffn with Q8_K activations for every projection: each token row
 * is quantised once for gate/up, each SwiGLU activation once for down. */
void haro_moe_ffn_q8k(const uint8_t *w_gate, const uint8_t *w_up, const uint8_t *w_down,
                      const uint8_t *sh_gate, const uint8_t *sh_up, const uint8_t *sh_down,
                      const float *sh_gate_inp, int64_t E, int64_t H, int64_t I,
                      int64_t T, int k, const float *x, const int32_t *ids,
                      const float *weights, int add_residual, float *y, int threads);

/* ---- a12: Q4_K quantiser (this project's own test-input generator) ------ */
/* Per 32-value group j: lo = min(0, min x), hi = max x; scale_j = (hi-lo)/15,
 * off_j = -lo.  d = f16(max scale/63), dmin = f16(max off/63); sc_j, m_j =
 * clamp(rint(scale_j/d)), clamp(rint(off_j/dmin)) in [0,63]; q = clamp(rint(
 * (x + dmin*m_j) / (d*sc_j)), 0, 15). Packed in the GGUF 144-byte layout. */
void haro_q4k_quantize_row(const float *x, int64_t k, uint8_t *out);

/* ---- seeded synthetic inputs --------------------------------------------- */
/* har/crates/har-serve/src/q4k.rs:109-120 */
void haro_lcg_values(int64_t count, uint64_t seed, float *out);
/* Counter-based normal: value i = mean + std * z_i, z from Box-Muller on two
 * splitmix64 words of (seed, i/2); index-addressable so any slice can be
 * generated independently (the device generator uses the same formula). */
void haro_normal_f32(uint64_t seed, int64_t start, int64_t count, float mean,
                     float std, float *out);
/* N(mean, std) rows quantised to Q4_K: `rows` rows of k values, element
 * (r, c) is normal index (row0 + r)*k + c of `seed`. */
void haro_gen_q4k_rows(uint64_t seed, int64_t row0, int64_t rows, int64_t k,
                       float mean, float std, uint8_t *out);
/* Zipf(s) top-k distinct routing over E experts: rank r (1-based) has
 * weight r^-s; ranks map to expert ids through a seeded permutation so hot
 * experts do not cluster on one expert-parallel shard; weights are a softmax
 * over seeded N(0,1) logits of the k selected (f64, rounded to f32). */
void haro_zipf_routing(uint64_t seed, int64_t T, int E, int k, double s,
                       int32_t *ids, float *weights);

/* utilities */
int haro_online_cpus(void);

#ifdef __cplusplus
}
#endif
#endif
