/*
 * TEST INFRASTRUCTURE ONLY -- the CPU oracle for the Magnetar CUDA provider's hot path.
 *
 * A plain-C restatement of the reference provider's operator semantics, following the
 * reference's one-thread-per-output CUDA kernels (src/kernels.cu), which themselves port
 * the reference CPU executor's operation order.  Only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / --impl reference legs may load it: it is the checker and the
 * timed CPU baseline, never the product path.
 *
 * Parity pin: the half-precision conversions are pinned by the reference's own exhaustive
 * 65,536-pattern round-trip tests and literal fixtures (src/half_precision.rs:127-163,
 * src/tests_conformance.rs:2349-2423); the closed-form known answers of
 * src/tests_conformance.rs:807-914 pin the matmul and attention edge cases.  The f32 ops
 * whose reference expectations come only from the absent CPU crate are "parity unpinned"
 * beyond those closed forms: the oracle recomputes them from the kernel semantics.
 */
#ifndef MAGNETAR_ORACLE_H
#define MAGNETAR_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Threads used by the OpenMP-parallel loops (0 = OpenMP default). */
void orc_set_threads(int threads);
int orc_get_threads(void);

/* ---- half precision (src/half_precision.rs:14-125, src/kernels.cu:2806-2911) ---- */
float orc_f16_to_f32(uint16_t bits);
float orc_bf16_to_f32(uint16_t bits);
uint16_t orc_f32_to_f16(float value);
uint16_t orc_f32_to_bf16(float value);
/* dtype: 1 = f16, 2 = bf16 */
void orc_encode_half(const float* in, uint16_t* out, uint64_t n, int dtype);
void orc_decode_half(const uint16_t* in, float* out, uint64_t n, int dtype);
/* dtype: 1 = f16, 2 = bf16.  op: 0 = add, 1 = mul (src/kernels.cu:2913-2939). */
void orc_half_binary(const uint16_t* a, const uint16_t* b, uint16_t* out, uint64_t n, int dtype, int op);
/* The executor's f32-resident form (src/executor.rs:1970-2013): encode both f32 inputs,
 * run the half op, decode the result back to f32. */
void orc_half_binary_f32(const float* a, const float* b, float* out, uint64_t n, int dtype, int op);

/* ---- elementwise (src/kernels.cu:30-117, 1091-1096) ---- */
void orc_add(const float* a, const float* b, float* out, uint64_t n);
void orc_bias_add(const float* a, const float* bias, float* out, uint64_t cols, uint64_t n);
void orc_mul(const float* a, const float* b, float* out, uint64_t n);
void orc_mul_scalar(const float* a, const float* b, float* out, uint64_t n);
void orc_scale(const float* x, float* out, float factor, uint64_t n);
void orc_silu(const float* x, float* out, uint64_t n);
void orc_gelu_tanh(const float* x, float* out, uint64_t n);
void orc_sigmoid(const float* x, float* out, uint64_t n);
void orc_softcap(const float* x, float* out, float cap, uint64_t n);
void orc_row_scale(const float* x, const float* scale, float* out, uint64_t rows, uint64_t cols);
void orc_q8_0_dequantize(const uint8_t* blocks, uint64_t rows, uint64_t cols, int transposed, float* out);
int64_t orc_greedy_select(const float* row, uint64_t cols, const uint64_t* ranges, uint32_t count, float temperature);
void orc_concat_heads(const float* a, const float* b, float* out, uint64_t rows, uint64_t heads, uint64_t a_width,
                      uint64_t b_width, uint64_t b_heads);
void orc_batched_matmul(const float* a, const float* b, float* out, uint64_t rows, uint64_t groups, uint64_t k,
                        uint64_t n, int transpose_b);
void orc_silu_mul(const float* gate, const float* up, float* out, uint64_t n);

/* ---- embedding (src/kernels.cu:127-176); returns 1 when an id was invalid ---- */
int orc_embedding(const float* table, const float* ids, float* out, uint64_t dim, uint64_t num_ids,
                  uint64_t vocab);

/* ---- rmsnorm (src/kernels.cu:1103-1138); weight may be NULL ---- */
void orc_rmsnorm(const float* x, const float* weight, float* out, uint64_t rows, uint64_t cols,
                 uint64_t weight_row_stride, float epsilon);

/* ---- rope (src/kernels.cu:1147-1229) ---- */
typedef struct orc_rope_params {
    float base, scale;
    uint64_t dimension, position_offset, head_count;
    uint32_t half_split;
    float banded_factor, low_freq_factor, high_freq_factor, original_context_length;
    uint64_t rotated_pairs;
    float yarn_factor, yarn_low, yarn_high, amplitude;
} orc_rope_params;
void orc_rope(const float* x, float* out, uint64_t rows, uint64_t cols, const orc_rope_params* p);

/* ---- softmax rows (src/kernels.cu:1232-1260); returns 1 when a row max is non-finite ---- */
int orc_softmax_rows(const float* x, float* out, uint64_t rows, uint64_t cols);

/* ---- matmul (src/kernels.cu:1265-1294, addend modes of :1351-1391) ---- */
void orc_matmul(const float* a, const float* b, float* out, uint64_t m, uint64_t k, uint64_t n,
                int transpose_a, int transpose_b, const float* addend, int addend_mode);
/* gated matmul: silu(a.g) * (a.u), src/kernels.cu:1517-1577 */
void orc_gated_matmul(const float* a, const float* gate, const float* up, float* out, uint64_t m,
                      uint64_t k, uint64_t n, int transpose_a, int transpose_b);

/* ---- attention (src/kernels.cu:1873-1959) ---- */
typedef struct orc_attention_params {
    uint64_t seq_len, kv_seq_len, head_count, kv_head_count, head_dimension;
    uint64_t q_model_dim, kv_model_dim;
    int causal;
    int64_t window_size; /* -1: no window */
    uint64_t query_position_offset;
    float score_scale; /* 0: 1/sqrt(head_dimension) */
    uint64_t value_dimension, v_model_dim;
} orc_attention_params;
void orc_attention(const float* q, const float* k, const float* v, float* out,
                   const orc_attention_params* p);

#ifdef __cplusplus
}
#endif

#endif
