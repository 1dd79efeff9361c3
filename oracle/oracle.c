/*
 * TEST INFRASTRUCTURE ONLY -- CPU oracle of the Magnetar CUDA provider's hot path.
 * See oracle.h for what pins each function.  Every function restates the reference
 * provider's kernel of the cited src/kernels.cu lines (one output per loop iteration, the
 * same f32 operations in the same order), parallelised over independent outputs with
 * OpenMP so that it can also serve as the timed CPU baseline.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static int g_threads = 0;

void orc_set_threads(int threads) {
    g_threads = threads;
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#endif
}

int orc_get_threads(void) {
#ifdef _OPENMP
    return g_threads > 0 ? g_threads : omp_get_max_threads();
#else
    return 1;
#endif
}

static inline float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* ------------------------------------------------------------------------------------ */
/* half precision: src/half_precision.rs:14-125 (identical to src/kernels.cu:2806-2911)   */
/* ------------------------------------------------------------------------------------ */

/* src/half_precision.rs:15-39 */
float orc_f16_to_f32(uint16_t bits) {
    uint32_t sign = ((uint32_t)(bits >> 15)) << 31;
    uint32_t exponent = (bits >> 10) & 0x1Fu;
    uint32_t mantissa = bits & 0x3FFu;
    uint32_t magnitude;
    if (exponent == 0) {
        if (mantissa == 0) {
            magnitude = 0;
        } else {
            /* subnormal: normalise the mantissa */
            uint32_t shift = 0;
            while ((mantissa & 0x400u) == 0) { mantissa <<= 1; shift++; }
            mantissa &= 0x3FFu;
            magnitude = ((127u - 15u - shift + 1u) << 23) | (mantissa << 13);
        }
    } else if (exponent == 0x1F) {
        magnitude = (0xFFu << 23) | (mantissa << 13);
    } else {
        magnitude = ((exponent - 15u + 127u) << 23) | (mantissa << 13);
    }
    return bits_f32(sign | magnitude);
}

/* src/half_precision.rs:42-44 */
float orc_bf16_to_f32(uint16_t bits) { return bits_f32((uint32_t)bits << 16); }

/* src/half_precision.rs:48-103: round to nearest, ties to even; NaN keeps its top payload
 * bits (a zero payload becomes 1). */
uint16_t orc_f32_to_f16(float value) {
    uint32_t bits = f32_bits(value);
    uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
    uint32_t man = bits & 0x007FFFFFu;
    int exp = (int)((bits >> 23) & 0xFFu);
    if (exp == 0xFF) {
        if (man == 0) return sign | 0x7C00u;
        uint16_t payload = (uint16_t)(man >> 13);
        return sign | 0x7C00u | (payload ? payload : 1u);
    }
    int unbiased = exp - 127;
    if (unbiased > 15) return sign | 0x7C00u;
    if (unbiased < -14) {
        uint32_t significand = exp == 0 ? man : (man | 0x00800000u);
        if (significand == 0) return sign;
        uint32_t shift = (uint32_t)(-(unbiased + 1));
        if (shift >= 32) return sign;
        uint32_t half = 1u << (shift - 1), mask = (1u << shift) - 1u;
        uint32_t result = significand >> shift, rem = significand & mask;
        if (rem > half || (rem == half && (result & 1u))) result++;
        return sign | (uint16_t)result;
    }
    uint32_t m10 = man >> 13, rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (m10 & 1u))) m10++;
    uint32_t exp16 = (uint32_t)(unbiased + 15);
    if (m10 == 0x400u) {
        if (exp16 + 1 >= 0x1Fu) return sign | 0x7C00u;
        return sign | (uint16_t)((exp16 + 1) << 10);
    }
    return sign | (uint16_t)((exp16 << 10) | m10);
}

/* src/half_precision.rs:107-117 */
uint16_t orc_f32_to_bf16(float value) {
    uint32_t bits = f32_bits(value);
    if (((bits >> 23) & 0xFFu) == 0xFFu && (bits & 0x007FFFFFu) != 0) {
        uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
        uint16_t m7 = (uint16_t)((bits >> 16) & 0x7Fu);
        return sign | 0x7F80u | (m7 ? m7 : 0x40u);
    }
    uint32_t rounded = bits + 0x7FFFu + ((bits >> 16) & 1u);
    return (uint16_t)(rounded >> 16);
}

/* The half kernels run their f32 add/mul on the GPU, whose f32 arithmetic returns the
 * canonical NaN 0x7FFFFFFF for any NaN result; x86 would propagate an input payload
 * instead, so the oracle canonicalises to model the device the reference runs on. */
static inline float device_nan_canonical(float v) {
    return v != v ? bits_f32(0x7FFFFFFFu) : v;
}

static inline float half_decode(uint16_t bits, int dtype) {
    return dtype == 1 ? orc_f16_to_f32(bits) : orc_bf16_to_f32(bits);
}
static inline uint16_t half_encode(float v, int dtype) {
    return dtype == 1 ? orc_f32_to_f16(v) : orc_f32_to_bf16(v);
}

/* Array forms of the conversions (bit patterns pass through unchanged, NaN payloads too). */
void orc_encode_half(const float* in, uint16_t* out, uint64_t n, int dtype) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; i++) out[i] = half_encode(in[i], dtype);
}

void orc_decode_half(const uint16_t* in, float* out, uint64_t n, int dtype) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; i++) out[i] = half_decode(in[i], dtype);
}

/* src/kernels.cu:2913-2939 */
void orc_half_binary(const uint16_t* a, const uint16_t* b, uint16_t* out, uint64_t n, int dtype, int op) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; i++) {
        float x = half_decode(a[i], dtype), y = half_decode(b[i], dtype);
        float r = op == 0 ? x + y : x * y;
        out[i] = half_encode(device_nan_canonical(r), dtype);
    }
}

/* src/executor.rs:1970-2013 with src/tests_conformance.rs:2333-2346 (half_expected) */
void orc_half_binary_f32(const float* a, const float* b, float* out, uint64_t n, int dtype, int op) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; i++) {
        float x = half_decode(half_encode(a[i], dtype), dtype);
        float y = half_decode(half_encode(b[i], dtype), dtype);
        float r = op == 0 ? x + y : x * y;
        out[i] = half_decode(half_encode(device_nan_canonical(r), dtype), dtype);
    }
}

/* ------------------------------------------------------------------------------------ */
/* elementwise                                                                           */
/* ------------------------------------------------------------------------------------ */

/* src/kernels.cu:30-35 */
void orc_add(const float* a, const float* b, float* out, uint64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; i++) out[i] = a[i] + b[i];
}

/* src/kernels.cu:1091-1096 */
void orc_bias_add(const float* a, const float* bias, float* out, uint64_t cols, uint64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; i++) out[i] = a[i] + bias[(uint64_t)i % cols];
}

/* src/kernels.cu:55-60 */
void orc_mul(const float* a, const float* b, float* out, uint64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; i++) out[i] = a[i] * b[i];
}

/* src/kernels.cu:112-117 */
void orc_mul_scalar(const float* a, const float* b, float* out, uint64_t n) {
    const float s = b[0];
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; i++) out[i] = a[i] * s;
}

/* src/kernels.cu:95-100 */
void orc_scale(const float* x, float* out, float factor, uint64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; i++) out[i] = x[i] * factor;
}

/* src/kernels.cu:73-79 */
void orc_silu(const float* x, float* out, uint64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; i++) {
        float v = x[i];
        out[i] = v * (1.0f / (1.0f + expf(-v)));
    }
}

/* src/kernels.cu:80-92: the tanh form of GELU, in the reference's order of operations */
void orc_gelu_tanh(const float* x, float* out, uint64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; i++) {
        float v = x[i];
        out[i] = 0.5f * v * (1.0f + tanhf(0.7978846f * (v + 0.044715f * v * v * v)));
    }
}

/* src/kernels.cu:1079-1084 */
void orc_sigmoid(const float* x, float* out, uint64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; i++) out[i] = 1.0f / (1.0f + expf(-x[i]));
}

/* src/kernels.cu:103-109 */
void orc_softcap(const float* x, float* out, float cap, uint64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; i++) out[i] = cap * tanhf(x[i] / cap);
}

/* Q8_0 blocks (src/kernels.rs:309-330, 1800-1838; src/kernels.cu:230-246): 34 bytes each, a
 * little-endian f16 scale d then 32 signed 8-bit quants q; value = q * d with d widened exactly.
 * out is the logical matrix: the stored [rows, cols] one, or its transpose when transposed. */
void orc_q8_0_dequantize(const uint8_t* blocks, uint64_t rows, uint64_t cols, int transposed, float* out) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < (int64_t)rows; r++) {
        for (uint64_t c = 0; c < cols; c++) {
            const uint64_t index = (uint64_t)r * cols + c, block = index / 32;
            const uint8_t* b = blocks + block * 34;
            const float d = orc_f16_to_f32((uint16_t)(b[0] | (b[1] << 8)));
            const float v = (float)(int8_t)b[2 + index % 32] * d;
            if (transposed) out[c * rows + (uint64_t)r] = v;
            else out[index] = v;
        }
    }
}

/* Host greedy selection (src/tests_conformance.rs:571-587, the Runtime's rule the device kernel
 * src/kernels.cu:1808-1866 matches): the first column, in column order, whose finite raw score,
 * outside every excluded [start, end) pair, divided by the temperature (as is when 0), is
 * strictly greater than every earlier one.  Returns -1 when no column is eligible. */
int64_t orc_greedy_select(const float* row, uint64_t cols, const uint64_t* ranges, uint32_t count, float temperature) {
    int64_t best = -1;
    float best_value = 0.0f;
    for (uint64_t c = 0; c < cols; c++) {
        const float raw = row[c];
        if (!isfinite(raw)) continue;
        int excluded = 0;
        for (uint32_t r = 0; r < count && !excluded; r++) excluded = c >= ranges[2 * r] && c < ranges[2 * r + 1];
        if (excluded) continue;
        const float score = temperature == 0.0f ? raw : raw / temperature;
        if (best < 0 || score > best_value) {
            best = (int64_t)c;
            best_value = score;
        }
    }
    return best;
}

/* src/kernels.cu:1066-1077: out[i] = x[i] * scale[i / cols] */
void orc_row_scale(const float* x, const float* scale, float* out, uint64_t rows, uint64_t cols) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)(rows * cols); i++) out[i] = x[i] * scale[(uint64_t)i / cols];
}

/* src/kernels.cu:5786-5812: head h of output row r = a's head h, then b's head h (or b's only
 * head when b_heads == 1) */
void orc_concat_heads(const float* a, const float* b, float* out, uint64_t rows, uint64_t heads, uint64_t a_width,
                      uint64_t b_width, uint64_t b_heads) {
    const uint64_t width = a_width + b_width;
#pragma omp parallel for schedule(static)
    for (int64_t idx = 0; idx < (int64_t)(rows * heads * width); idx++) {
        const uint64_t row = (uint64_t)idx / (heads * width), rem = (uint64_t)idx % (heads * width);
        const uint64_t head = rem / width, j = rem % width;
        out[idx] = j < a_width ? a[(row * heads + head) * a_width + j]
                               : b[(row * b_heads + (b_heads == 1 ? 0 : head)) * b_width + (j - a_width)];
    }
}

/* src/kernels.cu:6296-6336: out[r][g n + j] = sum over i in order of a[r][g k + i] times
 * b[g k + i][j] (or b[g n + j][i] with transpose_b) */
void orc_batched_matmul(const float* a, const float* b, float* out, uint64_t rows, uint64_t groups, uint64_t k,
                        uint64_t n, int transpose_b) {
    const uint64_t width = groups * n;
#pragma omp parallel for schedule(static)
    for (int64_t idx = 0; idx < (int64_t)(rows * width); idx++) {
        const uint64_t r = (uint64_t)idx / width, col = (uint64_t)idx % width, g = col / n, j = col % n;
        const float* in = a + r * groups * k + g * k;
        float sum = 0.0f;
        if (transpose_b) {
            const float* w = b + (g * n + j) * k;
            for (uint64_t i = 0; i < k; i++) sum += in[i] * w[i];
        } else {
            const float* w = b + g * k * n + j;
            for (uint64_t i = 0; i < k; i++) sum += in[i] * w[i * n];
        }
        out[idx] = sum;
    }
}

/* src/kernels.cu:64-71 */
void orc_silu_mul(const float* gate, const float* up, float* out, uint64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; i++) {
        float v = gate[i];
        float activated = v * (1.0f / (1.0f + expf(-v)));
        out[i] = activated * up[i];
    }
}

/* ------------------------------------------------------------------------------------ */
/* embedding: src/kernels.cu:127-176 (f32 table path)                                    */
/* ------------------------------------------------------------------------------------ */
int orc_embedding(const float* table, const float* ids, float* out, uint64_t dim, uint64_t num_ids,
                  uint64_t vocab) {
    int invalid = 0;
#pragma omp parallel for schedule(static) reduction(| : invalid)
    for (int64_t row = 0; row < (int64_t)num_ids; row++) {
        float raw = ids[row];
        /* negative, non-integer (NaN included) or >= vocab: the row stays unwritten */
        if (raw < 0.0f || raw != floorf(raw) || !((double)raw < (double)vocab)) {
            invalid = 1;
            continue;
        }
        uint64_t id = (uint64_t)raw;
        memcpy(out + (uint64_t)row * dim, table + id * dim, dim * sizeof(float));
    }
    return invalid;
}

/* ------------------------------------------------------------------------------------ */
/* rmsnorm: src/kernels.cu:1103-1138                                                      */
/* The reference sums squares in 256 strided slices, then a fixed-order tree; the oracle */
/* keeps exactly that order so that its sum is the reference kernel's.                   */
/* ------------------------------------------------------------------------------------ */
#define ORC_RMSNORM_THREADS 256
void orc_rmsnorm(const float* x, const float* weight, float* out, uint64_t rows, uint64_t cols,
                 uint64_t weight_row_stride, float epsilon) {
#pragma omp parallel for schedule(static)
    for (int64_t row = 0; row < (int64_t)rows; row++) {
        const float* in = x + (uint64_t)row * cols;
        const float* w = weight ? weight + (uint64_t)row * weight_row_stride : NULL;
        float partial[ORC_RMSNORM_THREADS];
        for (int t = 0; t < ORC_RMSNORM_THREADS; t++) {
            float s = 0.0f;
            for (uint64_t i = (uint64_t)t; i < cols; i += ORC_RMSNORM_THREADS) s += in[i] * in[i];
            partial[t] = s;
        }
        for (int stride = ORC_RMSNORM_THREADS / 2; stride > 0; stride /= 2)
            for (int t = 0; t < stride; t++) partial[t] += partial[t + stride];
        float scale = 1.0f / sqrtf(partial[0] / (float)cols + epsilon);
        float* o = out + (uint64_t)row * cols;
        for (uint64_t i = 0; i < cols; i++) o[i] = w ? in[i] * scale * w[i] : in[i] * scale;
    }
}

/* ------------------------------------------------------------------------------------ */
/* rope: src/kernels.cu:1147-1229 (one output pair per iteration; untouched columns of a */
/* partial-dimension block are copied, src/kernels.rs:4317-4322)                         */
/* ------------------------------------------------------------------------------------ */
void orc_rope(const float* x, float* out, uint64_t rows, uint64_t cols, const orc_rope_params* p) {
    const uint64_t head_width = cols / p->head_count;
    const uint64_t half = p->dimension / 2;
    if (p->dimension != head_width) memcpy(out, x, rows * cols * sizeof(float));
#pragma omp parallel for schedule(static)
    for (int64_t row = 0; row < (int64_t)rows; row++) {
        float position = (float)(p->position_offset + (uint64_t)row) * p->scale;
        for (uint64_t pair = 0; pair < half; pair++) {
            float frequency = powf(p->base, -2.0f * (float)pair / (float)p->dimension);
            if (p->banded_factor > 0.0f) {
                float wavelength = 6.283185307179586f / frequency;
                if (wavelength < p->original_context_length / p->high_freq_factor) {
                } else if (wavelength > p->original_context_length / p->low_freq_factor) {
                    frequency = frequency / p->banded_factor;
                } else {
                    float smooth = (p->original_context_length / wavelength - p->low_freq_factor) /
                                   (p->high_freq_factor - p->low_freq_factor);
                    frequency = (1.0f - smooth) * frequency / p->banded_factor + smooth * frequency;
                }
            }
            if (p->yarn_factor > 0.0f) {
                float high = p->yarn_low == p->yarn_high ? p->yarn_high + 0.001f : p->yarn_high;
                float ramp = ((float)pair - p->yarn_low) / (high - p->yarn_low);
                ramp = fminf(fmaxf(ramp, 0.0f), 1.0f);
                float interpolated = frequency / p->yarn_factor;
                frequency = interpolated * ramp + frequency * (1.0f - ramp);
            }
            float angle = pair < p->rotated_pairs ? position * frequency : 0.0f;
            float amp = pair < p->rotated_pairs ? p->amplitude : 1.0f;
            float s = sinf(angle) * amp, c = cosf(angle) * amp;
            for (uint64_t head = 0; head < p->head_count; head++) {
                uint64_t base = (uint64_t)row * cols + head * head_width;
                uint64_t first = p->half_split ? base + pair : base + 2 * pair;
                uint64_t second = p->half_split ? base + pair + half : base + 2 * pair + 1;
                float a = x[first], b = x[second];
                out[first] = a * c - b * s;
                out[second] = a * s + b * c;
            }
        }
    }
}

/* ------------------------------------------------------------------------------------ */
/* softmax rows: src/kernels.cu:1232-1260                                                 */
/* ------------------------------------------------------------------------------------ */
int orc_softmax_rows(const float* x, float* out, uint64_t rows, uint64_t cols) {
    int flag = 0;
#pragma omp parallel for schedule(static) reduction(| : flag)
    for (int64_t row = 0; row < (int64_t)rows; row++) {
        const float* in = x + (uint64_t)row * cols;
        float* o = out + (uint64_t)row * cols;
        float mx = -INFINITY;
        for (uint64_t i = 0; i < cols; i++) mx = fmaxf(mx, in[i]);
        if (!isfinite(mx)) {
            flag = 1;
            memset(o, 0, cols * sizeof(float));
            continue;
        }
        float sum = 0.0f;
        for (uint64_t i = 0; i < cols; i++) sum += expf(in[i] - mx);
        for (uint64_t i = 0; i < cols; i++) o[i] = expf(in[i] - mx) / sum;
    }
    return flag;
}

/* ------------------------------------------------------------------------------------ */
/* matmul: src/kernels.cu:1265-1294 -- each output accumulates k ascending in f32.       */
/* addend_mode 1 adds addend[col], 2 adds addend[row*n+col] after the sum                */
/* (src/kernels.cu:1382-1388).  The non-transposed loop nest keeps the per-output k      */
/* order while vectorising across columns.                                                */
/* ------------------------------------------------------------------------------------ */
void orc_matmul(const float* a, const float* b, float* out, uint64_t m, uint64_t k, uint64_t n,
                int transpose_a, int transpose_b, const float* addend, int addend_mode) {
    const uint64_t a_row_stride = transpose_a ? 1 : k, a_inner_stride = transpose_a ? m : 1;
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t row = 0; row < (int64_t)m; row++) {
        float* o = out + (uint64_t)row * n;
        const float* ar = a + (uint64_t)row * a_row_stride;
        if (!transpose_b) {
            for (uint64_t j = 0; j < n; j++) o[j] = 0.0f;
            for (uint64_t inner = 0; inner < k; inner++) {
                const float av = ar[inner * a_inner_stride];
                const float* br = b + inner * n;
                for (uint64_t j = 0; j < n; j++) o[j] += av * br[j];
            }
        } else {
            for (uint64_t j = 0; j < n; j++) {
                const float* bc = b + j * k;
                float acc = 0.0f;
                for (uint64_t inner = 0; inner < k; inner++) acc += ar[inner * a_inner_stride] * bc[inner];
                o[j] = acc;
            }
        }
        if (addend_mode == 1) {
            for (uint64_t j = 0; j < n; j++) o[j] += addend[j];
        } else if (addend_mode == 2) {
            for (uint64_t j = 0; j < n; j++) o[j] += addend[(uint64_t)row * n + j];
        }
    }
}

/* src/kernels.rs gated_matmul: bit-identical to two matmuls followed by silu_mul */
void orc_gated_matmul(const float* a, const float* gate, const float* up, float* out, uint64_t m,
                      uint64_t k, uint64_t n, int transpose_a, int transpose_b) {
    float* g = (float*)malloc(m * n * sizeof(float));
    float* u = (float*)malloc(m * n * sizeof(float));
    orc_matmul(a, gate, g, m, k, n, transpose_a, transpose_b, NULL, 0);
    orc_matmul(a, up, u, m, k, n, transpose_a, transpose_b, NULL, 0);
    orc_silu_mul(g, u, out, m * n);
    free(g);
    free(u);
}

/* ------------------------------------------------------------------------------------ */
/* attention: src/kernels.cu:1873-1959 -- per (head, query): max pass, sum-of-exp pass,  */
/* then the output as sum of normalised weights times V.  The scores are computed once   */
/* and reused (recomputing them, as the reference does, yields the same values).         */
/* ------------------------------------------------------------------------------------ */
void orc_attention(const float* q, const float* k, const float* v, float* out,
                   const orc_attention_params* p) {
    const uint64_t group = p->head_count / p->kv_head_count;
    const float scale = p->score_scale > 0.0f ? p->score_scale : 1.0f / sqrtf((float)p->head_dimension);
    const int64_t total = (int64_t)(p->head_count * p->seq_len);
#pragma omp parallel
    {
        float* scores = (float*)malloc((p->kv_seq_len + 1) * sizeof(float));
#pragma omp for schedule(dynamic, 4)
        for (int64_t idx = 0; idx < total; idx++) {
            uint64_t head = (uint64_t)idx / p->seq_len;
            uint64_t qi = (uint64_t)idx % p->seq_len;
            uint64_t kv_head = head / group;
            uint64_t qpos = p->query_position_offset + qi;
            uint64_t upper = p->causal ? qpos + 1 : p->kv_seq_len;
            uint64_t lower = 0;
            if (p->window_size >= 0) {
                uint64_t w = (uint64_t)p->window_size;
                uint64_t back = w > 0 ? w - 1 : 0;
                lower = qpos > back ? qpos - back : 0;
                if (lower > upper) lower = upper;
            }
            const float* qr = q + qi * p->q_model_dim + head * p->head_dimension;
            float mx = -INFINITY;
            for (uint64_t key = lower; key < upper; key++) {
                const float* kr = k + key * p->kv_model_dim + kv_head * p->head_dimension;
                float dot = 0.0f;
                for (uint64_t d = 0; d < p->head_dimension; d++) dot += qr[d] * kr[d];
                scores[key - lower] = dot * scale;
                mx = fmaxf(mx, dot * scale);
            }
            float sum = 0.0f;
            for (uint64_t key = lower; key < upper; key++) sum += expf(scores[key - lower] - mx);
            float* o = out + (qi * p->head_count + head) * p->value_dimension;
            for (uint64_t d = 0; d < p->value_dimension; d++) o[d] = 0.0f;
            for (uint64_t key = lower; key < upper; key++) {
                float weight = expf(scores[key - lower] - mx) / sum;
                const float* vr = v + key * p->v_model_dim + kv_head * p->value_dimension;
                for (uint64_t d = 0; d < p->value_dimension; d++) o[d] += weight * vr[d];
            }
        }
        free(scores);
    }
}
