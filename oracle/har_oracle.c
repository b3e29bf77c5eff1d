/*
 * har_oracle.c — CPU restatement of HAR's Q4_K MoE-FFN path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the product): loaded by
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg.
 * Build: oracle/Makefile (-O2 -ffp-contract=off, no -ffast-math).
 * Every function cites the reference file:line it restates; paths are
 * relative to the leoinfer/remora-lab repository root.
 */
#define _GNU_SOURCE
#include "har_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#if defined(__FP_FAST_FMAF) && !defined(HARO_ALLOW_FMA)
/* -ffp-contract=off keeps a*b+c as two roundings, as Rust does. */
#endif

/* ------------------------------------------------------------------------ */
/* a1                                                                        */
/* ------------------------------------------------------------------------ */

/* har/crates/har-serve/src/q4k.rs:22-50 */
float haro_f16_to_f32(uint8_t b0, uint8_t b1) {
    uint16_t bits = (uint16_t)(b0 | ((uint16_t)b1 << 8));
    uint32_t sign = (bits >> 15) & 1u;
    uint32_t ex = (bits >> 10) & 0x1fu;
    uint32_t frac = bits & 0x3ffu;
    float value;
    if (ex == 0) {
        if (frac == 0) {
            value = 0.0f;
        } else {
            float m = (float)frac / 1024.0f;
            value = m * ldexpf(1.0f, -14); /* 2f32.powi(-14), exact */
        }
    } else if (ex == 31) {
        value = frac == 0 ? INFINITY : NAN;
    } else {
        float m = 1.0f + (float)frac / 1024.0f;
        value = m * ldexpf(1.0f, (int)ex - 15);
    }
    return sign == 1 ? -value : value;
}

/* har/crates/har-demo/src/bin/har-native-qwen3.rs:116-136 */
float haro_half_to_f32(uint16_t value) {
    uint32_t sign = ((uint32_t)(value & 0x8000u)) << 16;
    uint32_t exponent = (value >> 10) & 0x1fu;
    uint32_t fraction = value & 0x03ffu;
    uint32_t bits;
    if (exponent == 0 && fraction == 0) {
        bits = sign;
    } else if (exponent == 0) {
        uint32_t mantissa = fraction, shift = 0;
        while ((mantissa & 0x0400u) == 0) {
            mantissa <<= 1;
            shift += 1;
        }
        mantissa &= 0x03ffu;
        bits = sign | ((127u - 14u - shift) << 23) | (mantissa << 13);
    } else if (exponent == 31) {
        bits = sign | 0x7f800000u | (fraction << 13);
    } else {
        bits = sign | ((exponent + 112u) << 23) | (fraction << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* IEEE binary32 -> binary16, round to nearest, ties to even. */
uint16_t haro_f32_to_f16_rne(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ex = (x >> 23) & 0xffu;
    uint32_t man = x & 0x7fffffu;
    if (ex == 0xff) /* Inf / NaN */
        return (uint16_t)(sign | 0x7c00u | (man ? 0x200u : 0u));
    int32_t e = (int32_t)ex - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u); /* overflow -> Inf */
    if (e <= 0) {
        /* subnormal half (or zero): value = man24 * 2^(ex-150); half unit 2^-24 */
        if (e < -10) return (uint16_t)sign;
        uint32_t m24 = man | 0x800000u;
        uint32_t shift = (uint32_t)(14 - e); /* bits to drop: 13 + (1 - e) */
        uint32_t q = m24 >> shift;
        uint32_t rem = m24 & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1u))) q += 1;
        return (uint16_t)(sign | q);
    }
    uint32_t q = ((uint32_t)e << 10) | (man >> 13);
    uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q += 1; /* may carry into Inf: correct */
    return (uint16_t)(sign | q);
}

/* ------------------------------------------------------------------------ */
/* a2 / a3                                                                   */
/* ------------------------------------------------------------------------ */

/* har/crates/har-serve/src/q4k.rs:60-66 */
uint32_t haro_scale_at(const uint8_t *block, int index) {
    if (index < 4) return (uint32_t)block[4 + index] & 63u;
    return ((uint32_t)block[4 + index + 4] & 15u) |
           (((uint32_t)block[4 + index - 4] >> 6) << 4);
}

/* har/crates/har-serve/src/q4k.rs:68-74 */
uint32_t haro_min_at(const uint8_t *block, int index) {
    if (index < 4) return (uint32_t)block[4 + index + 4] & 63u;
    return ((uint32_t)block[4 + index + 4] >> 4) |
           (((uint32_t)block[4 + index] >> 6) << 4);
}

/* har/crates/har-demo/src/bin/har-native-qwen3.rs:138-147 */
void haro_scale_min(const uint8_t *scales, int index, uint8_t *sc, uint8_t *m) {
    if (index < 4) {
        *sc = scales[index] & 63;
        *m = scales[index + 4] & 63;
    } else {
        *sc = (uint8_t)((scales[index + 4] & 15) | ((scales[index - 4] >> 6) << 4));
        *m = (uint8_t)((scales[index + 4] >> 4) | ((scales[index] >> 6) << 4));
    }
}

/* har/crates/har-serve/src/q4k.rs:77-89 */
float haro_q4k_dequant(const uint8_t *block, int index) {
    int group = index / 32;
    int lane_in_64 = index & 63;
    uint8_t q_byte = block[16 + (index / 64) * 32 + (lane_in_64 & 31)];
    uint8_t q = lane_in_64 < 32 ? (q_byte & 15) : (q_byte >> 4);
    float d = haro_f16_to_f32(block[0], block[1]);
    float dm = haro_f16_to_f32(block[2], block[3]);
    return d * (float)haro_scale_at(block, group) * (float)q -
           dm * (float)haro_min_at(block, group);
}

/* har/crates/har-demo/src/bin/har-native-qwen3.rs:1067-1093 */
void haro_decode_q4k_block(const uint8_t *block, float out[256]) {
    float d = haro_half_to_f32((uint16_t)(block[0] | (block[1] << 8)));
    float min = haro_half_to_f32((uint16_t)(block[2] | (block[3] << 8)));
    const uint8_t *scales = block + 4;
    int q_offset = 16, scale_index = 0;
    for (int base = 0; base < HARO_QK_K; base += 64) {
        uint8_t s1, m1, s2, m2;
        haro_scale_min(scales, scale_index, &s1, &m1);
        haro_scale_min(scales, scale_index + 1, &s2, &m2);
        for (int lane = 0; lane < 32; ++lane) {
            out[base + lane] = d * (float)s1 * (float)(block[q_offset + lane] & 0x0f) -
                               min * (float)m1;
            out[base + 32 + lane] = d * (float)s2 * (float)(block[q_offset + lane] >> 4) -
                                    min * (float)m2;
        }
        q_offset += 32;
        scale_index += 2;
    }
}

/* ------------------------------------------------------------------------ */
/* a4                                                                        */
/* ------------------------------------------------------------------------ */

/* har/crates/har-serve/src/q4k.rs:170-188 */
void haro_q4k_matvec(const uint8_t *w, int64_t rows, int64_t dim, const float *x,
                     float *out) {
    int64_t bpr = dim / HARO_QK_K;
    for (int64_t r = 0; r < rows; ++r) {
        float acc = 0.0f;
        for (int64_t b = 0; b < bpr; ++b) {
            const uint8_t *block = w + (r * bpr + b) * HARO_Q4K_BLOCK_BYTES;
            for (int i = 0; i < HARO_QK_K; ++i)
                acc += haro_q4k_dequant(block, i) * x[b * HARO_QK_K + i];
        }
        out[r] = acc;
    }
}

/* ------------------------------------------------------------------------ */
/* a5                                                                        */
/* ------------------------------------------------------------------------ */

/* har/crates/har-demo/src/bin/har-native-qwen3.rs:149-172 */
float haro_q4k_dot(const uint8_t *block, const float *input) {
    float d = haro_half_to_f32((uint16_t)(block[0] | (block[1] << 8)));
    float min = haro_half_to_f32((uint16_t)(block[2] | (block[3] << 8)));
    const uint8_t *scales = block + 4;
    int q_offset = 16, scale_index = 0;
    float sum = 0.0f;
    for (int input_base = 0; input_base < HARO_QK_K; input_base += 64) {
        uint8_t s1, m1, s2, m2;
        haro_scale_min(scales, scale_index, &s1, &m1);
        haro_scale_min(scales, scale_index + 1, &s2, &m2);
        float d1 = d * (float)s1;
        float d2 = d * (float)s2;
        float min1 = min * (float)m1;
        float min2 = min * (float)m2;
        for (int lane = 0; lane < 32; ++lane) {
            sum += (d1 * (float)(block[q_offset + lane] & 0x0f) - min1) * input[input_base + lane];
            sum += (d2 * (float)(block[q_offset + lane] >> 4) - min2) *
                   input[input_base + 32 + lane];
        }
        q_offset += 32;
        scale_index += 2;
    }
    return sum;
}

/* har/crates/har-demo/src/bin/har-native-qwen3.rs:207-232 (Q4_K arm) */
float haro_dot_quant_row(const uint8_t *row, const float *input, int64_t k) {
    float sum = 0.0f;
    for (int64_t b = 0; b < k / HARO_QK_K; ++b)
        sum += haro_q4k_dot(row + b * HARO_Q4K_BLOCK_BYTES, input + b * HARO_QK_K);
    return sum;
}

/* har/crates/har-demo/src/bin/har-native-qwen3.rs:174-205: one Q6_K block
 * (ql[128] @0, qh[64] @128, int8 scales[16] @192, f16 d @208) against 256
 * inputs, with q6k_dot's operation order: per (half, lane) the four terms
 * s*q*x summed left to right, times d, added to one f32 sum. */
float haro_q6k_dot(const uint8_t *block, const float *input) {
    const uint8_t *ql = block, *qh = block + 128, *scales = block + 192;
    const float d = haro_half_to_f32((uint16_t)(block[208] | (block[209] << 8)));
    float sum = 0.0f;
    for (int half = 0; half < 2; ++half) {
        const int ql_base = half * 64, qh_base = half * 32, scale_base = half * 8;
        const int input_base = half * 128;
        for (int lane = 0; lane < 32; ++lane) {
            const uint8_t high = qh[qh_base + lane];
            const uint8_t low_0 = ql[ql_base + lane];
            const uint8_t low_1 = ql[ql_base + 32 + lane];
            const int16_t q1 = (int16_t)((low_0 & 0x0f) | ((high & 0x03) << 4)) - 32;
            const int16_t q2 = (int16_t)((low_1 & 0x0f) | (((high >> 2) & 0x03) << 4)) - 32;
            const int16_t q3 = (int16_t)((low_0 >> 4) | (((high >> 4) & 0x03) << 4)) - 32;
            const int16_t q4 = (int16_t)((low_1 >> 4) | (((high >> 6) & 0x03) << 4)) - 32;
            const float s1 = (float)(int8_t)scales[scale_base + lane / 16];
            const float s2 = (float)(int8_t)scales[scale_base + lane / 16 + 2];
            const float s3 = (float)(int8_t)scales[scale_base + lane / 16 + 4];
            const float s4 = (float)(int8_t)scales[scale_base + lane / 16 + 6];
            sum += d * (s1 * (float)q1 * input[input_base + lane] +
                        s2 * (float)q2 * input[input_base + 32 + lane] +
                        s3 * (float)q3 * input[input_base + 64 + lane] +
                        s4 * (float)q4 * input[input_base + 96 + lane]);
        }
    }
    return sum;
}

/* har/crates/har-demo/src/bin/har-native-qwen3.rs:207-232 (Q6_K arm): the
 * row sum adds the per-block sums in block order. */
float haro_dot_quant_row_q6k(const uint8_t *row, const float *input, int64_t k) {
    float sum = 0.0f;
    for (int64_t b = 0; b < k / HARO_QK_K; ++b)
        sum += haro_q6k_dot(row + b * HARO_Q6K_BLOCK_BYTES, input + b * HARO_QK_K);
    return sum;
}

/* ---- Q3_K (f3; parity unpinned: the reference holds only the geometry,
 * har/crates/har-model/src/lib.rs:591; the layout restated is GGUF's, as
 * ggml's k-quants define it) ------------------------------------------------ */

/* 16 six-bit scales in 12 bytes: the low four bits of scale s sit in byte
 * s (s < 8, low nibble) or byte s - 8 (high nibble); its top two bits in
 * byte 8 + s % 4 at bit 2 * (s / 4). */
int haro_q3k_scale(const uint8_t *sc, int s) {
    const int low = s < 8 ? (sc[s] & 0x0f) : (sc[s - 8] >> 4);
    const int high = (sc[8 + (s & 3)] >> (2 * (s >> 2))) & 3;
    return low | (high << 4);
}

void haro_q3k_dequant_block(const uint8_t *block, float out[256]) {
    const uint8_t *hmask = block, *qs = block + 32, *sc = block + 96;
    const float d = haro_half_to_f32((uint16_t)(block[108] | (block[109] << 8)));
    for (int n = 0; n < 2; ++n)
        for (int j = 0; j < 4; ++j)
            for (int l = 0; l < 32; ++l) {
                const int s = 8 * n + 2 * j + l / 16;
                const float dl = d * (float)(haro_q3k_scale(sc, s) - 32);
                const int q2 = (qs[32 * n + l] >> (2 * j)) & 3;
                const int hi = (hmask[l] >> (4 * n + j)) & 1;
                out[128 * n + 32 * j + l] = dl * (float)(q2 - (hi ? 0 : 4));
            }
}

float haro_q3k_dot(const uint8_t *block, const float *input) {
    float w[256];
    haro_q3k_dequant_block(block, w);
    float sum = 0.0f;
    for (int i = 0; i < 256; ++i) sum += w[i] * input[i];
    return sum;
}

void haro_q3k_matvec(const uint8_t *w, int64_t rows, int64_t k, const float *x, float *out) {
    const int64_t rb = k / HARO_QK_K * HARO_Q3K_BLOCK_BYTES;
    for (int64_t r = 0; r < rows; ++r) {
        float sum = 0.0f;
        for (int64_t b = 0; b < k / HARO_QK_K; ++b)
            sum += haro_q3k_dot(w + r * rb + b * HARO_Q3K_BLOCK_BYTES, x + b * HARO_QK_K);
        out[r] = sum;
    }
}

/* matvec over a Q6_K tensor's rows (har-native-qwen35moe.rs:561-624 with
 * dot_row's Q6_K arm, :551-556): out[r] = dot_quant_row(row r, x). */
void haro_q6k_matvec(const uint8_t *w, int64_t rows, int64_t k, const float *x, float *out) {
    const int64_t rb = k / HARO_QK_K * HARO_Q6K_BLOCK_BYTES;
    for (int64_t r = 0; r < rows; ++r) out[r] = haro_dot_quant_row_q6k(w + r * rb, x, k);
}

/* har/crates/har-demo/src/bin/har-native-qwen35moe.rs:154-163 */
float haro_dot_f32_row(const float *row, const float *input, int64_t k) {
    float sum = 0.0f;
    for (int64_t i = 0; i < k; ++i) sum += row[i] * input[i];
    return sum;
}

/* har/crates/har-demo/src/bin/har-native-qwen35moe.rs:1168-1172: routed_moe's
 * router logits, self.matvec(ffn_gate_inp) on an F32 tensor [E][H]; each row
 * is dot_f32_row (:154-163).  The worker split of matvec (:583-624) only
 * decides which thread computes a row, not the row's value. */
void haro_router_logits(const float *gate_inp, int64_t E, int64_t H, const float *x,
                        float *logits) {
    for (int64_t e = 0; e < E; ++e) logits[e] = haro_dot_f32_row(gate_inp + e * H, x, H);
}

/* ------------------------------------------------------------------------ */
/* a6: expert_matvec with per-call worker threads                            */
/* ------------------------------------------------------------------------ */

int haro_online_cpus(void) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

typedef struct {
    const uint8_t *base;
    int64_t row_bytes, K, row_start, rows;
    const float *x;
    float *y;
} haro_rows_job;

/* har/crates/har-demo/src/bin/har-native-qwen35moe.rs:561-581 (matvec_rows) */
static void *haro_rows_worker(void *arg) {
    haro_rows_job *j = (haro_rows_job *)arg;
    for (int64_t r = 0; r < j->rows; ++r)
        j->y[r] = haro_dot_quant_row(j->base + (j->row_start + r) * j->row_bytes, j->x, j->K);
    return NULL;
}

static void haro_matvec_threads(const uint8_t *base, int64_t N, int64_t K, const float *x,
                                float *y, int threads) {
    int64_t row_bytes = K / HARO_QK_K * HARO_Q4K_BLOCK_BYTES;
    int64_t workers = threads > 0 ? threads : haro_online_cpus();
    if (workers > N) workers = N > 0 ? N : 1;
    int64_t chunk = (N + workers - 1) / workers; /* rows.div_ceil(workers) */
    if (workers <= 1) {
        haro_rows_job j = {base, row_bytes, K, 0, N, x, y};
        haro_rows_worker(&j);
        return;
    }
    pthread_t tid[256];
    haro_rows_job jobs[256];
    int64_t nj = 0;
    for (int64_t start = 0; start < N && nj < 256; start += chunk, ++nj) {
        int64_t n = (start + chunk <= N) ? chunk : N - start;
        jobs[nj] = (haro_rows_job){base, row_bytes, K, start, n, x, y + start};
        if (pthread_create(&tid[nj], NULL, haro_rows_worker, &jobs[nj]) != 0) {
            haro_rows_worker(&jobs[nj]);
            tid[nj] = 0;
        }
    }
    for (int64_t i = 0; i < nj; ++i)
        if (tid[i]) pthread_join(tid[i], NULL);
}

/* har/crates/har-demo/src/bin/har-native-qwen35moe.rs:626-689 */
void haro_expert_matvec(const uint8_t *tensor, int64_t E, int64_t N, int64_t K,
                        int64_t expert, const float *x, float *y, int threads) {
    (void)E;
    int64_t row_bytes = K / HARO_QK_K * HARO_Q4K_BLOCK_BYTES;
    haro_matvec_threads(tensor + expert * N * row_bytes, N, K, x, y, threads);
}

/* ------------------------------------------------------------------------ */
/* a7                                                                        */
/* ------------------------------------------------------------------------ */

/* har/crates/har-demo/src/bin/har-native-qwen35moe.rs:203-205 */
float haro_silu(float value) { return value / (1.0f + expf(-value)); }

/* har/crates/har-demo/src/bin/har-native-qwen35moe.rs:207-214 */
float haro_sigmoid(float value) {
    if (value >= 0.0f) return 1.0f / (1.0f + expf(-value));
    float e = expf(value);
    return e / (1.0f + e);
}

/* har/crates/har-demo/src/bin/har-native-qwen35moe.rs:979-1048 */
void haro_compose_moe_route(const uint8_t *w_gate, const uint8_t *w_up,
                            const uint8_t *w_down, const uint8_t *sh_gate,
                            const uint8_t *sh_up, const uint8_t *sh_down,
                            const float *sh_gate_inp, int64_t E, int64_t H,
                            int64_t I, int k, const float *input,
                            const int32_t *experts, const float *weights,
                            float *routed, int threads) {
    float *gate = (float *)malloc(sizeof(float) * (size_t)I);
    float *up = (float *)malloc(sizeof(float) * (size_t)I);
    float *down = (float *)malloc(sizeof(float) * (size_t)H);
    for (int64_t i = 0; i < H; ++i) routed[i] = 0.0f;
    for (int s = 0; s < k; ++s) {
        int64_t expert = experts[s];
        float weight = weights[s];
        haro_expert_matvec(w_gate, E, I, H, expert, input, gate, threads);
        haro_expert_matvec(w_up, E, I, H, expert, input, up, threads);
        for (int64_t i = 0; i < I; ++i) gate[i] = haro_silu(gate[i]) * up[i];
        haro_expert_matvec(w_down, E, H, I, expert, gate, down, threads);
        for (int64_t i = 0; i < H; ++i) routed[i] += weight * down[i];
    }
    if (sh_gate && sh_up && sh_down) {
        haro_matvec_threads(sh_gate, I, H, input, gate, threads);
        haro_matvec_threads(sh_up, I, H, input, up, threads);
        for (int64_t i = 0; i < I; ++i) gate[i] = haro_silu(gate[i]) * up[i];
        haro_matvec_threads(sh_down, H, I, gate, down, threads);
        float g = sh_gate_inp ? haro_sigmoid(haro_dot_f32_row(sh_gate_inp, input, H)) : 1.0f;
        for (int64_t i = 0; i < H; ++i) routed[i] += g * down[i];
    }
    free(gate);
    free(up);
    free(down);
}

void haro_moe_ffn(const uint8_t *w_gate, const uint8_t *w_up, const uint8_t *w_down,
                  const uint8_t *sh_gate, const uint8_t *sh_up, const uint8_t *sh_down,
                  const float *sh_gate_inp, int64_t E, int64_t H, int64_t I,
                  int64_t T, int k, const float *x, const int32_t *ids,
                  const float *weights, int add_residual, float *y, int threads) {
    for (int64_t t = 0; t < T; ++t) {
        haro_compose_moe_route(w_gate, w_up, w_down, sh_gate, sh_up, sh_down, sh_gate_inp,
                               E, H, I, k, x + t * H, ids + t * k, weights + t * k,
                               y + t * H, threads);
        if (add_residual) /* har-native-qwen35moe.rs:1152-1155: left + right */
            for (int64_t i = 0; i < H; ++i) y[t * H + i] = x[t * H + i] + y[t * H + i];
    }
}

/* ------------------------------------------------------------------------ */
/* a8                                                                        */
/* ------------------------------------------------------------------------ */

/* exp used by the router softmax.  Mode 0 (default) is glibc's expf, the
 * function Rust's f32::exp calls on Linux, so the oracle reproduces the
 * reference bit for bit.  glibc's expf is not correctly rounded: on 97,052
 * of the 1,120,927,745 floats in [-104, -0] it returns the neighbour of the
 * correctly rounded value.  Mode 1 rounds exp evaluated in double instead,
 * which is correctly rounded; the GPU router computes the same. */
static int haro_exp_mode = 0;
void haro_set_exp_mode(int mode) { haro_exp_mode = mode; }

/* glibc's expf restated (the function Rust's f32::exp calls): Szabolcs
 * Nagy's table-driven method, published in ARM's optimized-routines and used
 * by glibc since 2.28.  In double precision: k = round(x * 32/ln2) through
 * the 1.5 * 2^52 shift, r = x * 32/ln2 - k, exp(x) = 2^(k/32) * P(r) with
 * 2^(i/32) from a table (rounded to nearest double) and P a cubic with the
 * method's published coefficients; one rounding to float at the end.  On
 * x86-64 with FMA glibc runs the variant whose reduction and polynomial use
 * fused multiply-adds, which fma() restates here.  The device router
 * (expf_ref in the library) computes the same steps; haro_expf_mismatches
 * checks this function against the host's expf. */
static const uint64_t haro_exp2_i32[32] = {
    0x3ff0000000000000ull, 0x3ff059b0d3158574ull, 0x3ff0b5586cf9890full, 0x3ff11301d0125b51ull,
    0x3ff172b83c7d517bull, 0x3ff1d4873168b9aaull, 0x3ff2387a6e756238ull, 0x3ff29e9df51fdee1ull,
    0x3ff306fe0a31b715ull, 0x3ff371a7373aa9cbull, 0x3ff3dea64c123422ull, 0x3ff44e086061892dull,
    0x3ff4bfdad5362a27ull, 0x3ff5342b569d4f82ull, 0x3ff5ab07dd485429ull, 0x3ff6247eb03a5585ull,
    0x3ff6a09e667f3bcdull, 0x3ff71f75e8ec5f74ull, 0x3ff7a11473eb0187ull, 0x3ff82589994cce13ull,
    0x3ff8ace5422aa0dbull, 0x3ff93737b0cdc5e5ull, 0x3ff9c49182a3f090ull, 0x3ffa5503b23e255dull,
    0x3ffae89f995ad3adull, 0x3ffb7f76f2fb5e47ull, 0x3ffc199bdd85529cull, 0x3ffcb720dcef9069ull,
    0x3ffd5818dcfba487ull, 0x3ffdfc97337b9b5full, 0x3ffea4afa2a490daull, 0x3fff50765b6e4540ull};

void haro_exp2_table(uint64_t *out) { memcpy(out, haro_exp2_i32, sizeof(haro_exp2_i32)); }

float haro_expf_restated(float x) {
    if (x < -0x1.9fe368p6f) return 0.0f;      /* below log(2^-150) */
    if (x > 0x1.62e42ep6f) return INFINITY;    /* above log(2^128) */
    const double inv = 0x1.71547652b82fep+0 * 32.0, shift = 0x1.8p+52;
    const double c0 = 0x1.c6af84b912394p-5 / 32768.0, c1 = 0x1.ebfce50fac4f3p-3 / 1024.0,
                 c2 = 0x1.62e42ff0c52d6p-1 / 32.0;
    const double xd = (double)x;
    double kd = fma(inv, xd, shift);
    uint64_t ki;
    memcpy(&ki, &kd, 8);
    kd -= shift;
    const double r = fma(inv, xd, -kd);
    const uint32_t i = (uint32_t)(ki & 31u);
    const uint64_t sb = haro_exp2_i32[i] + ((ki - i) << 47);
    double sd;
    memcpy(&sd, &sb, 8);
    const double q = fma(c0, r, c1);
    const double r2 = r * r;
    double y = fma(c2, r, 1.0);
    y = fma(q, r2, y);
    return (float)(y * sd);
}

/* Floats with bit patterns lo..hi (inclusive, walked upward) where the
 * restatement and the host's expf differ; *first gets the first such pattern. */
uint64_t haro_expf_mismatches(uint32_t lo, uint32_t hi, uint32_t *first) {
    uint64_t bad = 0;
    for (uint32_t u = lo;; ++u) {
        float x, a, b;
        memcpy(&x, &u, 4);
        a = expf(x);
        b = haro_expf_restated(x);
        if (memcmp(&a, &b, 4) != 0) {
            if (!bad && first) *first = u;
            ++bad;
        }
        if (u == hi) break;
    }
    return bad;
}

static float haro_router_exp(float v) {
    if (haro_exp_mode == 1) return (float)exp((double)v);
    if (haro_exp_mode == 2) return haro_expf_restated(v);
    return expf(v);
}

/* f32::total_cmp(b, a) ordering then lower index (descending by p). Returns
 * nonzero when entry (pa, ia) sorts before (pb, ib). */
static int haro_before(float pa, int ia, float pb, int ib) {
    int32_t a, b;
    memcpy(&a, &pa, 4);
    memcpy(&b, &pb, 4);
    /* total order key of f32 (as Rust's total_cmp) */
    a ^= (int32_t)(((uint32_t)(a >> 31)) >> 1);
    b ^= (int32_t)(((uint32_t)(b >> 31)) >> 1);
    if (a != b) return a > b;
    return ia < ib;
}

/* har/crates/har-demo/src/bin/har-native-qwen35moe.rs:1167-1204 */
void haro_route_topk(const float *router, int E, int k, int32_t *ids, float *weights) {
    float max_router = -INFINITY;
    for (int i = 0; i < E; ++i) max_router = fmaxf(max_router, router[i]); /* f32::max */
    float *probs = (float *)malloc(sizeof(float) * (size_t)E);
    float denominator = 0.0f;
    for (int i = 0; i < E; ++i) {
        probs[i] = haro_router_exp(router[i] - max_router);
        denominator += probs[i];
    }
    denominator = fmaxf(denominator, HARO_ROUTER_EPS);
    for (int i = 0; i < E; ++i) probs[i] = probs[i] / denominator;
    /* The reference sorts all E then takes k; a k-pass selection with the
     * same strict order yields the same prefix. */
    unsigned char *taken = (unsigned char *)calloc((size_t)E, 1);
    for (int s = 0; s < k; ++s) {
        int best = -1;
        for (int i = 0; i < E; ++i) {
            if (taken[i]) continue;
            if (best < 0 || haro_before(probs[i], i, probs[best], best)) best = i;
        }
        taken[best] = 1;
        ids[s] = best;
    }
    float selected_total = 0.0f;
    for (int s = 0; s < k; ++s) selected_total += probs[ids[s]];
    selected_total = fmaxf(selected_total, HARO_ROUTER_EPS);
    for (int s = 0; s < k; ++s) weights[s] = probs[ids[s]] / selected_total;
    free(taken);
    free(probs);
}

/* ------------------------------------------------------------------------ */
/* a9                                                                        */
/* ------------------------------------------------------------------------ */

/* har/crates/har-serve/src/moe.rs:195-202 */
void haro_group_by_expert(int64_t T, int k, int E, const int32_t *ids, int32_t *counts,
                          int32_t *offsets, int32_t *order) {
    for (int e = 0; e < E; ++e) counts[e] = 0;
    for (int64_t i = 0; i < T * k; ++i) counts[ids[i]] += 1;
    offsets[0] = 0;
    for (int e = 0; e < E; ++e) offsets[e + 1] = offsets[e] + counts[e];
    int32_t *fill = (int32_t *)malloc(sizeof(int32_t) * (size_t)E);
    for (int e = 0; e < E; ++e) fill[e] = offsets[e];
    for (int64_t i = 0; i < T * k; ++i) order[fill[ids[i]]++] = (int32_t)i;
    free(fill);
}

/* ------------------------------------------------------------------------ */
/* a11: Q8_K                                                                 */
/* ------------------------------------------------------------------------ */

void haro_q8k_quantize(const float *x, int64_t k, uint8_t *out) {
    for (int64_t b = 0; b < k / HARO_QK_K; ++b) {
        const float *v = x + b * HARO_QK_K;
        uint8_t *blk = out + b * HARO_Q8K_BLOCK_BYTES;
        float amax = 0.0f;
        for (int i = 0; i < HARO_QK_K; ++i) amax = fmaxf(amax, fabsf(v[i]));
        float d = 0.0f;
        int8_t qs[256];
        if (amax == 0.0f) {
            memset(qs, 0, sizeof qs);
        } else {
            float iscale = 127.0f / amax;
            d = amax / 127.0f;
            /* amax below 127/FLT_MAX: 127/amax overflows, divide by d instead */
            int use_div = isinf(iscale);
            for (int i = 0; i < HARO_QK_K; ++i) {
                float t = use_div ? rintf(v[i] / d) : rintf(v[i] * iscale);
                int q = (int)t;
                if (q > 127) q = 127;
                if (q < -127) q = -127;
                qs[i] = (int8_t)q;
            }
        }
        memcpy(blk, &d, 4);
        memcpy(blk + 4, qs, 256);
        for (int g = 0; g < 16; ++g) {
            int16_t s = 0;
            for (int i = 0; i < 16; ++i) s = (int16_t)(s + qs[16 * g + i]);
            memcpy(blk + 260 + 2 * g, &s, 2);
        }
    }
}

float haro_q8k_dot_row(const uint8_t *row, const uint8_t *xq, int64_t k) {
    float sum = 0.0f;
    for (int64_t b = 0; b < k / HARO_QK_K; ++b) {
        const uint8_t *w = row + b * HARO_Q4K_BLOCK_BYTES;
        const uint8_t *a = xq + b * HARO_Q8K_BLOCK_BYTES;
        float dx;
        memcpy(&dx, a, 4);
        const int8_t *q8 = (const int8_t *)(a + 4);
        int16_t bs[16];
        memcpy(bs, a + 260, 32);
        float dw = haro_half_to_f32((uint16_t)(w[0] | (w[1] << 8)));
        float dmw = haro_half_to_f32((uint16_t)(w[2] | (w[3] << 8)));
        int32_t i1 = 0, i2 = 0;
        for (int c = 0; c < 4; ++c) { /* 64-value chunk: sub-blocks 2c (low) and 2c+1 (high) */
            uint8_t s1, m1, s2, m2;
            haro_scale_min(w + 4, 2 * c, &s1, &m1);
            haro_scale_min(w + 4, 2 * c + 1, &s2, &m2);
            int32_t lo = 0, hi = 0;
            for (int l = 0; l < 32; ++l) {
                uint8_t qb = w[16 + 32 * c + l];
                lo += (int32_t)(qb & 15) * q8[64 * c + l];
                hi += (int32_t)(qb >> 4) * q8[64 * c + 32 + l];
            }
            i1 += (int32_t)s1 * lo + (int32_t)s2 * hi;
            i2 += (int32_t)m1 * (bs[4 * c] + bs[4 * c + 1]) + (int32_t)m2 * (bs[4 * c + 2] + bs[4 * c + 3]);
        }
        float blk = (dw * dx) * (float)i1 - (dmw * dx) * (float)i2;
        sum += blk;
    }
    return sum;
}

void haro_q4k_gemv_q8k(const uint8_t *w, int64_t rows, int64_t k, const uint8_t *xq,
                       float *out) {
    int64_t row_bytes = k / HARO_QK_K * HARO_Q4K_BLOCK_BYTES;
    for (int64_t r = 0; r < rows; ++r) out[r] = haro_q8k_dot_row(w + r * row_bytes, xq, k);
}

void haro_moe_ffn_q8k(const uint8_t *w_gate, const uint8_t *w_up, const uint8_t *w_down,
                      const uint8_t *sh_gate, const uint8_t *sh_up, const uint8_t *sh_down,
                      const float *sh_gate_inp, int64_t E, int64_t H, int64_t I,
                      int64_t T, int k, const float *x, const int32_t *ids,
                      const float *weights, int add_residual, float *y, int threads) {
    (void)E;
    (void)threads;
    int64_t rb_h = H / HARO_QK_K * HARO_Q4K_BLOCK_BYTES; /* gate/up row bytes */
    int64_t rb_i = I / HARO_QK_K * HARO_Q4K_BLOCK_BYTES; /* down row bytes */
    uint8_t *xq = (uint8_t *)malloc((size_t)(H / HARO_QK_K * HARO_Q8K_BLOCK_BYTES));
    uint8_t *aq = (uint8_t *)malloc((size_t)(I / HARO_QK_K * HARO_Q8K_BLOCK_BYTES));
    float *g = (float *)malloc(sizeof(float) * (size_t)I);
    float *u = (float *)malloc(sizeof(float) * (size_t)I);
    float *dn = (float *)malloc(sizeof(float) * (size_t)H);
    for (int64_t t = 0; t < T; ++t) {
        const float *xt = x + t * H;
        float *yt = y + t * H;
        haro_q8k_quantize(xt, H, xq);
        for (int64_t i = 0; i < H; ++i) yt[i] = 0.0f;
        int nslot = k + ((sh_gate && sh_up && sh_down) ? 1 : 0);
        for (int s = 0; s < nslot; ++s) {
            const uint8_t *wg, *wu, *wd;
            float wt;
            if (s < k) {
                int64_t e = ids[t * k + s];
                wg = w_gate + e * I * rb_h;
                wu = w_up + e * I * rb_h;
                wd = w_down + e * H * rb_i;
                wt = weights[t * k + s];
            } else {
                wg = sh_gate;
                wu = sh_up;
                wd = sh_down;
                wt = sh_gate_inp ? haro_sigmoid(haro_dot_f32_row(sh_gate_inp, xt, H)) : 1.0f;
            }
            haro_q4k_gemv_q8k(wg, I, H, xq, g);
            haro_q4k_gemv_q8k(wu, I, H, xq, u);
            for (int64_t i = 0; i < I; ++i) g[i] = haro_silu(g[i]) * u[i];
            haro_q8k_quantize(g, I, aq);
            haro_q4k_gemv_q8k(wd, H, I, aq, dn);
            for (int64_t i = 0; i < H; ++i) yt[i] += wt * dn[i];
        }
        if (add_residual)
            for (int64_t i = 0; i < H; ++i) yt[i] = xt[i] + yt[i];
    }
    free(xq);
    free(aq);
    free(g);
    free(u);
    free(dn);
}

/* ------------------------------------------------------------------------ */
/* a12: Q4_K quantiser (own design)                                          */
/* ------------------------------------------------------------------------ */

static int haro_clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

static void haro_q4k_quantize_block(const float *x, uint8_t *out) {
    float scale[8], off[8];
    for (int j = 0; j < 8; ++j) {
        float lo = x[32 * j], hi = x[32 * j];
        for (int i = 1; i < 32; ++i) {
            lo = fminf(lo, x[32 * j + i]);
            hi = fmaxf(hi, x[32 * j + i]);
        }
        if (lo > 0.0f) lo = 0.0f;
        scale[j] = (hi - lo) / 15.0f;
        off[j] = -lo;
    }
    float smax = 0.0f, omax = 0.0f;
    for (int j = 0; j < 8; ++j) {
        smax = fmaxf(smax, scale[j]);
        omax = fmaxf(omax, off[j]);
    }
    uint16_t dh = haro_f32_to_f16_rne(smax / 63.0f);
    uint16_t mh = haro_f32_to_f16_rne(omax / 63.0f);
    float df = haro_half_to_f32(dh), mf = haro_half_to_f32(mh);
    int sc[8], mn[8];
    for (int j = 0; j < 8; ++j) {
        sc[j] = df > 0.0f ? haro_clampi((int)rintf(scale[j] / df), 0, 63) : 0;
        mn[j] = mf > 0.0f ? haro_clampi((int)rintf(off[j] / mf), 0, 63) : 0;
    }
    memset(out, 0, HARO_Q4K_BLOCK_BYTES);
    out[0] = (uint8_t)(dh & 0xff);
    out[1] = (uint8_t)(dh >> 8);
    out[2] = (uint8_t)(mh & 0xff);
    out[3] = (uint8_t)(mh >> 8);
    uint8_t *s = out + 4;
    for (int j = 0; j < 4; ++j) {
        s[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        s[j + 4] = (uint8_t)((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
        s[j + 8] = (uint8_t)((sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4));
    }
    for (int j = 0; j < 8; ++j) {
        float step = df * (float)sc[j];
        float bias = mf * (float)mn[j];
        for (int i = 0; i < 32; ++i) {
            int idx = 32 * j + i;
            int q = step > 0.0f ? haro_clampi((int)rintf((x[idx] + bias) / step), 0, 15) : 0;
            int byte = 16 + (idx / 64) * 32 + (idx & 31);
            if ((idx & 63) < 32)
                out[byte] = (uint8_t)((out[byte] & 0xf0) | q);
            else
                out[byte] = (uint8_t)((out[byte] & 0x0f) | (q << 4));
        }
    }
}

void haro_q4k_quantize_row(const float *x, int64_t k, uint8_t *out) {
    for (int64_t b = 0; b < k / HARO_QK_K; ++b)
        haro_q4k_quantize_block(x + b * HARO_QK_K, out + b * HARO_Q4K_BLOCK_BYTES);
}

/* ------------------------------------------------------------------------ */
/* generators                                                                */
/* ------------------------------------------------------------------------ */

/* har/crates/har-serve/src/q4k.rs:109-120 */
void haro_lcg_values(int64_t count, uint64_t seed, float *out) {
    uint64_t state = seed;
    for (int64_t i = 0; i < count; ++i) {
        state = state * 6364136223846793005ULL + 1442695040888963407ULL;
        float u = (float)(uint32_t)(state >> 40) / (float)(1u << 24);
        out[i] = u - 0.5f;
    }
}

static uint64_t haro_mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}

static double haro_normal_at(uint64_t seed, int64_t i) {
    uint64_t p = (uint64_t)(i >> 1);
    uint64_t base = seed * 0x9E3779B97F4A7C15ULL;
    uint64_t a = haro_mix64(base + 2 * p + 1);
    uint64_t b = haro_mix64(base + 2 * p + 2);
    double u1 = (double)((a >> 11) + 1) * (1.0 / 9007199254740992.0); /* (0, 1] */
    double u2 = (double)(b >> 11) * (1.0 / 9007199254740992.0);       /* [0, 1) */
    double r = sqrt(-2.0 * log(u1));
    double th = 6.283185307179586 * u2;
    return (i & 1) ? r * sin(th) : r * cos(th);
}

void haro_normal_f32(uint64_t seed, int64_t start, int64_t count, float mean, float std,
                     float *out) {
    for (int64_t i = 0; i < count; ++i)
        out[i] = (float)((double)mean + (double)std * haro_normal_at(seed, start + i));
}

void haro_gen_q4k_rows(uint64_t seed, int64_t row0, int64_t rows, int64_t k, float mean,
                       float std, uint8_t *out) {
    float *tmp = (float *)malloc(sizeof(float) * (size_t)k);
    int64_t rb = k / HARO_QK_K * HARO_Q4K_BLOCK_BYTES;
    for (int64_t r = 0; r < rows; ++r) {
        haro_normal_f32(seed, (row0 + r) * k, k, mean, std, tmp);
        haro_q4k_quantize_row(tmp, k, out + r * rb);
    }
    free(tmp);
}

void haro_zipf_routing(uint64_t seed, int64_t T, int E, int k, double s, int32_t *ids,
                       float *weights) {
    double *cdf = (double *)malloc(sizeof(double) * (size_t)E);
    int32_t *perm = (int32_t *)malloc(sizeof(int32_t) * (size_t)E);
    double acc = 0.0;
    for (int r = 0; r < E; ++r) {
        acc += pow((double)(r + 1), -s);
        cdf[r] = acc;
    }
    for (int r = 0; r < E; ++r) cdf[r] /= acc;
    for (int e = 0; e < E; ++e) perm[e] = e;
    uint64_t st = haro_mix64(seed ^ 0x5eedULL);
    for (int e = E - 1; e > 0; --e) { /* Fisher-Yates */
        st = haro_mix64(st + 0x9E3779B97F4A7C15ULL);
        int j = (int)(st % (uint64_t)(e + 1));
        int32_t t = perm[e];
        perm[e] = perm[j];
        perm[j] = t;
    }
    uint64_t ctr = 0;
    double lg[64];
    for (int64_t t = 0; t < T; ++t) {
        int got = 0;
        while (got < k) {
            uint64_t h = haro_mix64(seed * 0xD1B54A32D192ED03ULL + (ctr++));
            double u = (double)(h >> 11) * (1.0 / 9007199254740992.0);
            int lo = 0, hi = E - 1;
            while (lo < hi) {
                int mid = (lo + hi) / 2;
                if (cdf[mid] > u) hi = mid; else lo = mid + 1;
            }
            int32_t e = perm[lo];
            int dup = 0;
            for (int q = 0; q < got; ++q) dup |= ids[t * k + q] == e;
            if (!dup) ids[t * k + got++] = e;
        }
        double mx = -1e300, den = 0.0;
        for (int q = 0; q < k && q < 64; ++q) {
            lg[q] = haro_normal_at(seed ^ 0xA5A5A5A5ULL, t * k + q);
            if (lg[q] > mx) mx = lg[q];
        }
        for (int q = 0; q < k && q < 64; ++q) den += exp(lg[q] - mx);
        for (int q = 0; q < k && q < 64; ++q) weights[t * k + q] = (float)(exp(lg[q] - mx) / den);
    }
    free(cdf);
    free(perm);
}
