/*
 * magnetar_cuda.h -- C ABI of the B200 (sm_100a) CUDA execution provider for the Magnetar
 * runtime.  Drop-in for the operator path of astorise/Magnetar-provider-CUDA: the reference
 * serves the Runtime through the Rust trait `ProviderExecutionApi` implemented by
 * `CudaExecutor` (src/executor.rs:2244-2565) over launch wrappers `CudaKernels::<op>`
 * (src/kernels.rs:794-7132) that JIT-compile src/kernels.cu with NVRTC.  Here the kernels
 * are precompiled sm_100a code and every entry point below is a plain C function a Rust
 * `extern "C"` block binds directly.
 *
 * Conventions
 *  - Every function returns an mg_status; MG_OK is 0.  On failure the calling thread's
 *    mg_last_error() holds a redacted detail string (never a pointer or handle), mirroring
 *    CudaError{code, detail} (src/error.rs:49-52).
 *  - Work is stream-ordered on the device's stream; calls return after enqueue.  Only
 *    downloads and the data-dependent flag checks (embedding ids, softmax rows) wait for the
 *    device, as in the reference (src/kernels.rs:3984-3997, 4371-4378).
 *  - Op outputs follow the reference's output-offer rule (src/executor.rs:1276-1321): when
 *    *out is non-NULL and holds the output's dtype and element count it is written in place
 *    (its shape is set to the result's); otherwise a new buffer is allocated from the
 *    device's stream-ordered pool and returned in *out.
 */
#ifndef MAGNETAR_CUDA_H
#define MAGNETAR_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MG_ABI_VERSION 1
#define MG_MAX_RANK 8

/* Status codes.  1..9 mirror CudaErrorCode one-to-one (src/error.rs:14-42) so a Rust shim
 * maps them into KernelError exactly as src/error.rs:97-134 does; 10..13 are the
 * KernelError variants the executor raises itself (src/executor.rs:1422-2027). */
typedef enum mg_status {
    MG_OK = 0,
    MG_SHAPE_UNSUPPORTED = 1,      /* CudaErrorCode::ShapeUnsupported */
    MG_DTYPE_UNSUPPORTED = 2,      /* CudaErrorCode::DTypeUnsupported */
    MG_LAYOUT_UNSUPPORTED = 3,     /* CudaErrorCode::LayoutUnsupported */
    MG_EXECUTION_FAILED = 4,       /* CudaErrorCode::ExecutionFailed */
    MG_OUT_OF_DEVICE_MEMORY = 5,   /* CudaErrorCode::OutOfDeviceMemory */
    MG_COMPILATION_FAILED = 6,     /* CudaErrorCode::CompilationFailed (never raised: no JIT) */
    MG_DRIVER_FAILED = 7,          /* CudaErrorCode::DriverFailed */
    MG_DEVICE_UNAVAILABLE = 8,     /* CudaErrorCode::DeviceUnavailable */
    MG_CAPTURE_UNSUPPORTED = 9,    /* CudaErrorCode::CaptureUnsupported */
    MG_KERNEL_NOT_FOUND = 10,      /* KernelError::KernelNotFound */
    MG_ATTRIBUTE_UNSUPPORTED = 11, /* KernelError::KernelAttributeUnsupported */
    MG_INVALID_ARGUMENT = 12,      /* a NULL handle or out-parameter */
    MG_KERNEL_TIMEOUT = 13         /* KernelError::KernelTimeout (deadline_millis == 0) */
} mg_status;

/* Element types: f32 everywhere, f16/bf16 for add-half/mul-half
 * (CudaHalfDType, src/kernels.rs:211-215). */
/* MG_Q8_0: a packed weight (mg_buffer_upload_q8_0); only matmul's b, embedding's table,
 * mg_dequantize_q8 and downloads accept it. */
typedef enum mg_dtype { MG_F32 = 0, MG_F16 = 1, MG_BF16 = 2, MG_Q8_0 = 3 } mg_dtype;

typedef struct mg_device mg_device;     /* CudaKernels + its stream (src/kernels.rs:538-616) */
typedef struct mg_buffer mg_buffer;     /* CudaDeviceBuffer / CudaHalfBuffer (src/kernels.rs:211-276) */
typedef struct mg_executor mg_executor; /* CudaExecutor (src/executor.rs:91-118) */
typedef struct mg_comm mg_comm;         /* one rank of a tensor-parallel group (src/multi.rs) */

/* ---------------------------------------------------------------------------------- */
/* Library, errors                                                                     */
/* ---------------------------------------------------------------------------------- */
int mg_abi_version(void);
/* Detail of the calling thread's last failure ("" when none). */
const char* mg_last_error(void);
/* Human-readable name of a status ("ShapeUnsupported", ...). */
const char* mg_status_name(mg_status status);

/* ---------------------------------------------------------------------------------- */
/* Devices -- replaces CudaProvider::for_device + device discovery                     */
/* (src/provider.rs:119-192, src/device.rs:41-92)                                      */
/* ---------------------------------------------------------------------------------- */
typedef struct mg_device_info {
    int ordinal;
    char name[96];
    int sm_major, sm_minor; /* "sm_XY" */
    int sm_count;
    uint64_t total_bytes, free_bytes;
} mg_device_info;

/* Number of visible CUDA devices; 0 (and MG_OK) when no driver/device is present. */
mg_status mg_device_count(int* count);
/* Opens device `ordinal`: creates its stream and stream-ordered memory pool.  Returns
 * MG_DEVICE_UNAVAILABLE when there is no such device or it is not sm_100 (graceful
 * unavailability, src/provider.rs:149-192). */
mg_status mg_device_open(int ordinal, mg_device** out);
mg_status mg_device_close(mg_device* device);
mg_status mg_device_get_info(mg_device* device, mg_device_info* info);
/* Waits for all work on the device's stream. */
mg_status mg_device_synchronize(mg_device* device);
/* The device's cudaStream_t (as void*). */
void* mg_device_stream(mg_device* device);
/* Makes the device enqueue on `stream` (a cudaStream_t of the same device) instead of
 * its own; NULL restores its own stream. */
mg_status mg_device_set_stream(mg_device* device, void* stream);
/* Upload/download counters (src/kernels.rs:546-552, 1453-1466). */
mg_status mg_device_counters(mg_device* device, uint64_t* uploads, uint64_t* downloads);
/* Number of kernels this library has launched on the device since it was opened. */
uint64_t mg_device_launch_count(mg_device* device);

/* ---------------------------------------------------------------------------------- */
/* Buffers -- CudaKernels::{upload, upload_half, download, download_half,              */
/* download_rows, zeros} (src/kernels.rs:1630-1641, 2118-2171, 2118-2138)              */
/* ---------------------------------------------------------------------------------- */
mg_status mg_buffer_create(mg_device* device, mg_dtype dtype, int rank, const uint64_t* shape,
                           mg_buffer** out);
/* A zero-filled buffer set on the device, with no upload (src/kernels.rs zeros). */
mg_status mg_buffer_zeros(mg_device* device, mg_dtype dtype, int rank, const uint64_t* shape,
                          mg_buffer** out);
/* A non-owning view of caller-owned device memory (e.g. a framework tensor). */
mg_status mg_buffer_wrap(mg_device* device, mg_dtype dtype, int rank, const uint64_t* shape,
                         void* device_ptr, mg_buffer** out);
mg_status mg_buffer_release(mg_buffer* buffer);
/* Raw bytes in the buffer's own dtype: `bytes` must equal the buffer's byte size. */
mg_status mg_buffer_upload(mg_buffer* buffer, const void* host, uint64_t bytes);
mg_status mg_buffer_download(const mg_buffer* buffer, void* host, uint64_t bytes);
/* f32 host values, encoded on the device to the buffer's dtype with the reference's
 * round-to-nearest-even and NaN rules (src/half_precision.rs:48-117). */
mg_status mg_buffer_upload_f32(mg_buffer* buffer, const float* host, uint64_t count);
/* The buffer's values decoded to f32 on the host side of the call. */
mg_status mg_buffer_download_f32(const mg_buffer* buffer, float* host, uint64_t count);
/* Rows [first_row, first_row + rows) of a rank-2 f32 buffer (src/kernels.rs download_rows);
 * MG_SHAPE_UNSUPPORTED when the range is outside the buffer. */
mg_status mg_buffer_download_rows(const mg_buffer* buffer, uint64_t first_row, uint64_t rows,
                                  float* host, uint64_t count);
mg_status mg_buffer_shape(const mg_buffer* buffer, int* rank, uint64_t* shape /* [MG_MAX_RANK] */);
mg_status mg_buffer_dtype(const mg_buffer* buffer, mg_dtype* dtype);
mg_status mg_buffer_reshape(mg_buffer* buffer, int rank, const uint64_t* shape);
void* mg_buffer_device_ptr(const mg_buffer* buffer);
/* Marks a buffer as a weight (its contents change rarely): the tensor-core matmul then keeps
 * the buffer's K-major tf32 operand form after first use instead of re-deriving it on every
 * call, as the reference prepares compact weights at upload (src/kernels.rs:1667-1723).  Any
 * write to the buffer drops the prepared form. */
mg_status mg_buffer_set_weight(mg_buffer* buffer, int is_weight);
/* 1 when a weight holds its compact form: a matrix of at least 65536 values, all exactly
 * bfloat16, kept also as its bfloat16 bits, which the few-row (M <= 16) matmul streams instead
 * of the f32 values -- half the bytes, bit-identical results (the reference's compact weight,
 * `CudaDeviceBuffer::is_compact`, src/kernels.rs:257-268, 1668-1712).  Built and checked on the
 * first such matmul that reads the weight; 0 before that, for other buffers, and for null. */
int mg_buffer_is_compact(const mg_buffer* buffer); /* 1 for packed weights too, as the reference's */

/* Packed weights (`execute-direct-quantized-weights`).  Q8_0 only: 34-byte blocks of a
 * little-endian f16 scale and 32 signed 8-bit quants, `stored_rows` x `stored_cols` values in
 * stored row-major order (stored_cols a multiple of 32); the logical matrix is the stored one, or
 * its transpose when `transposed` (a checkpoint's [out, in] weight read as matmul B [in, out]).
 * Replaces CudaKernels::upload_packed_weight's Q8_0 branch (src/kernels.rs:1725-1838): the blocks
 * are split on the device into quants and f32 scales (the f16 widened exactly).  A matmul with a
 * transposed-storage Q8_0 b and at most 16 rows of a streams the quants (k a multiple of 128);
 * other matmuls dequantize b for the call; an embedding lookup reads the rows of a packed table
 * stored untransposed. */
#define MG_PACKED_Q8_0 0
mg_status mg_buffer_upload_q8_0(mg_device* d, const void* blocks, uint64_t bytes, uint64_t stored_rows,
                                uint64_t stored_cols, int transposed, mg_buffer** out);
/* 1 for a packed buffer (the reference's `is_q8()`, src/kernels.rs:376-378). */
int mg_buffer_is_q8(const mg_buffer* buffer);
/* A packed weight's logical matrix as f32 (src/kernels.rs:1964-1967). */
mg_status mg_dequantize_q8(mg_device* d, const mg_buffer* packed, mg_buffer** out);

/* ---------------------------------------------------------------------------------- */
/* Kernels -- one entry per advertised hot-path operator, with the validation of the    */
/* matching CudaKernels method.                                                          */
/* ---------------------------------------------------------------------------------- */

/* add: same shape, or b a [cols]/[1, cols] row broadcast over a (src/kernels.rs:2956-3015) */
mg_status mg_add(mg_device* d, const mg_buffer* a, const mg_buffer* b, mg_buffer** out);
/* mul: same shape, or b of shape [1] scaling every element (src/kernels.rs:3017-3037,
 * src/executor.rs:1917-1927) */
mg_status mg_mul(mg_device* d, const mg_buffer* a, const mg_buffer* b, mg_buffer** out);
/* residual-add: add's rules (src/kernels.rs:3039-3046) */
mg_status mg_residual_add(mg_device* d, const mg_buffer* input, const mg_buffer* residual,
                          mg_buffer** out);
/* x * factor (src/kernels.cu:95-100; embedding's `scale`) */
mg_status mg_scale(mg_device* d, const mg_buffer* x, float factor, mg_buffer** out);
/* silu(x) = x * (1 / (1 + exp(-x))) (src/kernels.rs:3103-3118) */
mg_status mg_silu(mg_device* d, const mg_buffer* x, mg_buffer** out);
/* silu(gate) * up (src/kernels.rs:4492-4523) */
mg_status mg_silu_mul(mg_device* d, const mg_buffer* gate, const mg_buffer* up, mg_buffer** out);
/* gelu, tanh approximation (src/kernels.rs:3167-3170, kernels.cu:80-92) */
mg_status mg_gelu_tanh(mg_device* d, const mg_buffer* x, mg_buffer** out);
/* activation kind sigmoid: 1 / (1 + exp(-x)) (src/kernels.rs:3121-3125) */
mg_status mg_sigmoid(mg_device* d, const mg_buffer* x, mg_buffer** out);
/* activation kind softcap: cap * tanh(x / cap); cap finite and positive (src/kernels.rs:3211-3224) */
mg_status mg_softcap(mg_device* d, const mg_buffer* x, float cap, mg_buffer** out);
/* row-scale: out[t, :] = x[t, :] * scale[t], x rank-2, scale [T] or [T, 1] (src/kernels.rs:3255-3290) */
mg_status mg_row_scale(mg_device* d, const mg_buffer* x, const mg_buffer* scale, mg_buffer** out);
/* concat along the first dimension; trailing dimensions must agree (src/kernels.rs:3058-3100) */
mg_status mg_concat(mg_device* d, const mg_buffer* a, const mg_buffer* b, mg_buffer** out);
/* concat across heads: row r = for each head h, a's head h then b's head h (second_head_count ==
 * head_count) or b's only head (second_head_count == 1) (src/kernels.rs:7084-7130) */
mg_status mg_concat_heads(mg_device* d, const mg_buffer* a, const mg_buffer* b, uint64_t head_count,
                          uint64_t second_head_count, mg_buffer** out);
/* batched-matmul: out [rows, groups * n], group g of row r = a[r, g k .. (g + 1) k] times
 * b[g k .. (g + 1) k, :] or, with transpose_b, times b[g n .. (g + 1) n, :] transposed
 * (src/kernels.rs:5882-5950) */
mg_status mg_batched_matmul(mg_device* d, const mg_buffer* a, const mg_buffer* b, uint64_t groups, int transpose_b,
                            mg_buffer** out);
/* Half-precision add/mul on f16 or bf16 buffers, bit-exact with the reference's integer
 * decode -> f32 op -> RNE encode (src/kernels.rs:2227-2266, src/kernels.cu:2806-2939).
 * Both inputs must share shape and dtype. */
mg_status mg_add_half(mg_device* d, const mg_buffer* a, const mg_buffer* b, mg_buffer** out);
mg_status mg_mul_half(mg_device* d, const mg_buffer* a, const mg_buffer* b, mg_buffer** out);
/* The executor's f32-resident form of add-half/mul-half (src/executor.rs:1970-2013):
 * f32 buffers in and out, each value passed through `dtype` exactly as the reference's
 * host round trip does, with no host traffic.  op: 0 add, 1 mul. */
mg_status mg_half_binary_f32(mg_device* d, const mg_buffer* a, const mg_buffer* b, mg_dtype dtype,
                             int op, mg_buffer** out);

/* embedding: rank-2 f32 table [vocab, dim], f32 ids holding integers; out [num_ids, dim].
 * An id that is negative, non-integer or >= vocab fails the call with
 * MG_SHAPE_UNSUPPORTED after the device reports it (src/kernels.rs:3833-3997).
 * has_scale != 0 multiplies the rows by `scale` (src/executor.rs:1502-1518). */
mg_status mg_embedding(mg_device* d, const mg_buffer* table, const mg_buffer* ids, int has_scale,
                       float scale, mg_buffer** out);

/* rmsnorm (src/kernels.rs:4013-4104): weight NULL for the scale-less form; weight [cols],
 * [1, cols], the input's shape or [rows, cols]; head_count/head_dimension both 0, or both
 * positive for per-head normalisation.  epsilon must be positive. */
mg_status mg_rmsnorm(mg_device* d, const mg_buffer* x, const mg_buffer* weight, float epsilon,
                     uint64_t head_count, uint64_t head_dimension, mg_buffer** out);

/* rope (src/kernels.rs:4224-4355).  pairing: 0 interleaved (2i, 2i+1), 1 half-split
 * (i, i + dimension/2).  banded_factor == 0 disables banded scaling; yarn_factor == 0
 * disables YaRN (yarn_low/high are the correction range, amplitude the attention factor);
 * rotated_pairs == UINT64_MAX rotates every pair. */
typedef struct mg_rope_params {
    float base;  /* default 10000 */
    float scale; /* default 1 */
    uint64_t dimension;
    uint64_t position_offset;
    uint64_t head_count; /* default 1 */
    int pairing;
    float banded_factor, low_freq_factor, high_freq_factor, original_context_length;
    uint64_t rotated_pairs;
    float yarn_factor, yarn_low, yarn_high, amplitude;
} mg_rope_params;
mg_status mg_rope(mg_device* d, const mg_buffer* x, const mg_rope_params* params, mg_buffer** out);

/* kv-write (src/kernels.rs:2278-2325, `append-kv-history-in-place`): writes the rows of the
 * rank-2 `rows` [count, width] over `store`'s rows row_offset .. row_offset + count, in place;
 * the store's other rows are unchanged.  Both f32 of the same width; a range past the store's
 * rows is MG_SHAPE_UNSUPPORTED. */
mg_status mg_kv_write(mg_device* d, mg_buffer* store, const mg_buffer* rows, uint64_t row_offset);

/* Greedy selection (src/kernels.rs:4441-4488, `keep-sampling-on-device`): the column of row `row`
 * of the logits (the last dimension's columns) with the highest score / temperature (the score as
 * is when temperature is 0), among columns whose raw score is finite and which lie outside each
 * of the `excluded_count` [start, end) pairs in `excluded` ([2 * count] uint64); ties, -0 against
 * +0 included, go to the lowest column.  *found = 0 when no column is eligible.  A row past the
 * logits is MG_SHAPE_UNSUPPORTED; it reads its result back (not capturable). */
mg_status mg_greedy_select(mg_device* d, const mg_buffer* logits, uint64_t row, const uint64_t* excluded,
                           uint32_t excluded_count, float temperature, int* found, uint64_t* column);

/* softmax over the rows of a rank-2 buffer; MG_EXECUTION_FAILED when a row has no finite
 * maximum (src/kernels.rs:4357-4386). */
mg_status mg_softmax(mg_device* d, const mg_buffer* x, mg_buffer** out);

/* matmul C = op(A) op(B) (+ addend), f32 (src/kernels.rs:4388-4436, 5518-5789).
 * Rank-2 operands; transpose flags as the reference's transpose_a/transpose_b. */
mg_status mg_matmul(mg_device* d, const mg_buffer* a, const mg_buffer* b, int transpose_a,
                    int transpose_b, mg_buffer** out);
/* matmul + bias row [n] or [1, n] (matmul-bias) */
mg_status mg_matmul_bias(mg_device* d, const mg_buffer* a, const mg_buffer* b, const mg_buffer* bias,
                         int transpose_a, int transpose_b, mg_buffer** out);
/* matmul + residual [m, n] (matmul-residual) */
mg_status mg_matmul_residual(mg_device* d, const mg_buffer* a, const mg_buffer* b,
                             const mg_buffer* residual, int transpose_a, int transpose_b,
                             mg_buffer** out);
/* matmul C[m, n] = A[m, k] B[k, n] for 1 <= m <= 16 that allocates nothing.
 * No counterpart in the reference: it is an extra entry point for callers that cannot
 * allocate device memory when they multiply -- a runtime whose device memory is already
 * fully handed out under a fixed budget, or a latency-critical thread that must not enter
 * the driver's allocator.  The caller owns a, b and out (row-major f32, b 16-byte aligned,
 * n a multiple of 4); the split-k partial sums live in a workspace compiled into the library,
 * MG_GEMV_FIXED_WORKSPACE_BYTES per GPU that loads it, held until the process exits.  A
 * shape whose partials need more than that fails with MG_SHAPE_UNSUPPORTED.  The first call
 * on a device looks up the workspace's address (make that first call before any stream
 * capture); calls on one device share the workspace, so calls that overlap on the GPU race.
 * `stream` is a cudaStream_t of device `device_ordinal` (NULL: the default stream). */
#define MG_GEMV_FIXED_WORKSPACE_BYTES (8u << 20)
mg_status mg_matmul_gemv_fixed(int device_ordinal, void* stream, const float* a, const float* b, float* out,
                               uint64_t m, uint64_t k, uint64_t n);
/* silu(A gate) * (A up) (gated-matmul, src/kernels.rs:4529-4917) */
mg_status mg_gated_matmul(mg_device* d, const mg_buffer* a, const mg_buffer* gate,
                          const mg_buffer* up, int transpose_a, int transpose_b, mg_buffer** out);

/* attention (src/kernels.rs:6505-6884): q [seq, heads*D], k [kv_rows, kv_heads*D],
 * v [kv_rows, kv_heads*Dv] -> out [seq, heads*Dv].  kv_head_count 0 = head_count;
 * value_dimension 0 = head_dimension; window_size < 0 = none (requires causal);
 * key_count < 0 = all kv rows; has_scale 0 = 1/sqrt(D). */
typedef struct mg_attention_params {
    uint64_t head_count;
    uint64_t head_dimension;
    uint64_t kv_head_count;
    uint64_t value_dimension;
    int64_t window_size;
    int causal;
    int64_t key_count;
    int has_scale;
    float scale;
} mg_attention_params;
mg_status mg_attention(mg_device* d, const mg_buffer* q, const mg_buffer* k, const mg_buffer* v,
                       const mg_attention_params* params, mg_buffer** out);

/* ---------------------------------------------------------------------------------- */
/* Executor -- ProviderExecutionApi over a tensor table keyed by resource id             */
/* (src/executor.rs:91-118, 1191-1321, 1422-2027, 2244-2565)                             */
/* ---------------------------------------------------------------------------------- */
typedef enum mg_attr_kind { MG_ATTR_INT = 0, MG_ATTR_FLOAT = 1, MG_ATTR_BOOL = 2, MG_ATTR_STRING = 3 } mg_attr_kind;

/* One OperatorAttributeValue (Integer | Float | Boolean | String). */
typedef struct mg_attribute {
    const char* name;
    int kind;
    int64_t int_value; /* MG_ATTR_INT, MG_ATTR_BOOL (0/1) */
    double float_value;
    const char* string_value;
} mg_attribute;

/* One KernelInvocation: kernel name, input resource ids (with each input's descriptor
 * dtype, NULL = all f32), one output id, attributes, deadline (-1 = none, 0 = already
 * expired -> MG_KERNEL_TIMEOUT, src/executor.rs:1202-1210). */
typedef struct mg_invocation {
    const char* kernel;
    int input_count;
    const char* const* inputs;
    const int* input_dtypes;
    const char* output;
    int attribute_count;
    const mg_attribute* attributes;
    int64_t deadline_millis;
} mg_invocation;

mg_status mg_executor_create(mg_device* device, mg_executor** out);
mg_status mg_executor_destroy(mg_executor* executor);
/* write_tensor / write_weight_tensor: HostTensor {shape, f32 data} (src/executor.rs:2339-2372).
 * Writing an id replaces (and frees) its previous buffer. */
mg_status mg_executor_write_tensor(mg_executor* ex, const char* id, int rank, const uint64_t* shape,
                                   const float* data);
mg_status mg_executor_write_weight_tensor(mg_executor* ex, const char* id, int rank,
                                          const uint64_t* shape, const float* data);
mg_status mg_executor_write_zeroed_tensor(mg_executor* ex, const char* id, int rank,
                                          const uint64_t* shape);
/* Binds an existing device buffer (not copied) as resource `id`; the executor takes
 * ownership of the handle. */
mg_status mg_executor_adopt_buffer(mg_executor* ex, const char* id, mg_buffer* buffer);
/* Borrowed handle of resource `id` (valid until it is rewritten or released). */
mg_status mg_executor_buffer(mg_executor* ex, const char* id, mg_buffer** out);
/* read_tensor: MG_SHAPE_UNSUPPORTED when `capacity` is too small, MG_EXECUTION_FAILED
 * when there is no such resource. */
mg_status mg_executor_read_tensor(mg_executor* ex, const char* id, float* data, uint64_t capacity,
                                  int* rank, uint64_t* shape);
mg_status mg_executor_read_tensor_rows(mg_executor* ex, const char* id, uint64_t first_row,
                                       uint64_t rows, float* data, uint64_t capacity);
/* write_packed_weight_tensor (src/executor.rs:404-420): `format` MG_PACKED_Q8_0; arguments as
 * mg_buffer_upload_q8_0.  MG_DTYPE_UNSUPPORTED for other formats. */
mg_status mg_executor_write_packed_weight_tensor(mg_executor* ex, const char* id, int format, const void* blocks,
                                                 uint64_t bytes, uint64_t stored_rows, uint64_t stored_cols,
                                                 int transposed);
/* select_greedy_column (src/executor.rs:2549-2563): mg_greedy_select over a resident tensor. */
mg_status mg_executor_select_greedy_column(mg_executor* ex, const char* id, uint64_t row, const uint64_t* excluded,
                                           uint32_t excluded_count, float temperature, int* found,
                                           uint64_t* column);
/* *released = 1 when a resource was dropped (src/executor.rs release_tensor). */
mg_status mg_executor_release_tensor(mg_executor* ex, const char* id, int* released);
/* *present = 0 when the id is not resident. */
mg_status mg_executor_resident_shape(mg_executor* ex, const char* id, int* present, int* rank,
                                     uint64_t* shape);
mg_status mg_executor_copy_tensor(mg_executor* ex, const char* from, const char* to);
/* submit_kernel + complete_kernel in one call: runs the invocation on the stream. */
mg_status mg_executor_submit_kernel(mg_executor* ex, const mg_invocation* invocation);
mg_status mg_executor_synchronize(mg_executor* ex);
/* Step capture (src/executor.rs:177-376): invocations between begin and end are recorded
 * into one CUDA graph, replayed by mg_executor_replay_step.  Invocations that need a host
 * read while captured (softmax) fail with MG_CAPTURE_UNSUPPORTED; embedding ids are
 * checked once the replayed step has run. */
mg_status mg_executor_begin_step_capture(mg_executor* ex);
mg_status mg_executor_end_step_capture(mg_executor* ex);
mg_status mg_executor_abort_step_capture(mg_executor* ex);
mg_status mg_executor_replay_step(mg_executor* ex);
/* `count` back-to-back replays, then one embedding-id check covering all of them (the flag
 * is sticky across replays and reset by the check). */
mg_status mg_executor_replay_steps(mg_executor* ex, int count);
/* One replay with no embedding-id check (the flag accumulates) ... */
mg_status mg_executor_launch_step(mg_executor* ex);
/* ... and the check of every replay since the last check (waits for the device). */
mg_status mg_executor_check_steps(mg_executor* ex);
/* Step capture with advancing attributes (src/kernels.rs:1019-1062, StepCaptureRequest's
 * advancing_attributes): while recording, a launch whose attribute is named here --
 * "position_offset" (rope), "key_count" (attention with a key count: one query row),
 * "row_offset" (kv-write) -- adds the replay's offset to that attribute at run time, and
 * records the largest offset it stays in bounds for.  mg_executor_replay_step_at replays at
 * an offset (above the captured bound: MG_CAPTURE_UNSUPPORTED, nothing runs); the other
 * replays use offset 0.  A decode loop captures one step and replays it at 0, 1, 2, ... */
mg_status mg_executor_begin_step_capture_advancing(mg_executor* ex, const char* const* attributes, int count);
mg_status mg_executor_replay_step_at(mg_executor* ex, uint64_t offset);
/* One replay with its host I/O (src/executor.rs replay_step(id, offset, inputs) followed by the
 * step's reads): each to_device entry's `bytes` are copied into the captured buffer of `id`
 * before the replay, each other entry's buffer is copied to `host` after it, and one
 * synchronisation covers them and the embedding-id check.  `bytes` must equal the buffer's. */
typedef struct mg_step_io {
    const char* id;
    void* host;
    uint64_t bytes;
    int to_device; /* 1: input written before the replay; 0: output read after it */
} mg_step_io;
mg_status mg_executor_replay_step_io(mg_executor* ex, uint64_t offset, const mg_step_io* io, int count);
/* The largest offset the captured step accepts (UINT64_MAX: unbounded). */
mg_status mg_executor_step_max_offset(mg_executor* ex, uint64_t* out);
/* Several captured steps per executor (src/executor.rs:209-340, StepCaptureId):
 * mg_executor_end_step_capture_id ends the capture in progress, keeps its graph under a new
 * id and runs it once (so the captured step's results are available, as end_step_capture
 * does there).  mg_executor_replay_capture is replay_step(id, offset, inputs) with the
 * outputs read in the same call (entries as mg_executor_replay_step_io): it refuses, with
 * MG_CAPTURE_UNSUPPORTED and nothing run, a step whose resources no longer have their
 * captured storage ("resource '...' no longer has its captured storage"), an input the step
 * never read, and an input the step reads through a weight's operand form; embedding ids
 * written to the step are checked on the host first (MG_SHAPE_UNSUPPORTED).
 * mg_executor_release_step_capture drops a step (src/executor.rs release_step_capture); an
 * unknown id is not an error.  Device memory a live step addresses is never freed under it:
 * a workspace that grows, a dropped operand form or a replaced tensor stays allocated until
 * the last step addressing it is released.  The single-step calls above replay the step
 * that mg_executor_end_step_capture made last. */
mg_status mg_executor_end_step_capture_id(mg_executor* ex, uint64_t* id);
mg_status mg_executor_replay_capture(mg_executor* ex, uint64_t id, uint64_t offset, const mg_step_io* io,
                                     int count);
mg_status mg_executor_release_step_capture(mg_executor* ex, uint64_t id);
/* Number of captured steps the executor holds. */
mg_status mg_executor_step_capture_count(mg_executor* ex, int* count);
/* Observation log (src/executor.rs:1082-1100): counts of Started/Completed/Failed. */
mg_status mg_executor_observations(mg_executor* ex, uint64_t* started, uint64_t* completed,
                                   uint64_t* failed);
/* The observation log itself (src/executor.rs:1082-1100, KernelObservation): the most recent
 * MG_OBSERVATION_LOG_CAPACITY events, oldest first.  Every submit records DispatchStarted,
 * then DispatchCompleted, DispatchFailed (with the status), or Timeout (an expired deadline);
 * an output the device cannot hold also records MemoryFeasibilityFailed before the failure.
 * `invocation` numbers the executor's submits from 0.  With out == NULL only *count is set;
 * a capacity below the count is MG_SHAPE_UNSUPPORTED. */
#define MG_OBSERVATION_LOG_CAPACITY 4096
typedef enum mg_observation_kind {
    MG_OBSERVATION_DISPATCH_STARTED = 0,
    MG_OBSERVATION_DISPATCH_COMPLETED = 1,
    MG_OBSERVATION_DISPATCH_FAILED = 2,
    MG_OBSERVATION_TIMEOUT = 3,
    MG_OBSERVATION_MEMORY_FEASIBILITY_FAILED = 4
} mg_observation_kind;
typedef struct mg_observation {
    int kind;          /* mg_observation_kind */
    char kernel[48];   /* the invocation's kernel name (truncated) */
    uint64_t invocation;
    int status;        /* mg_status of a failure (MG_OK otherwise) */
} mg_observation;
mg_status mg_executor_observation_log(mg_executor* ex, mg_observation* out, uint32_t capacity, uint32_t* count);

/* ---------------------------------------------------------------------------------- */
/* Tensor parallel -- src/multi.rs, src/multi/tensor_parallel.rs                        */
/* One process per GPU; ranks join an NCCL communicator from a 128-byte unique id.      */
/* ---------------------------------------------------------------------------------- */
#define MG_COMM_ID_BYTES 128
mg_status mg_comm_unique_id(unsigned char id[MG_COMM_ID_BYTES]);
mg_status mg_comm_init(mg_device* device, int rank, int world, const unsigned char id[MG_COMM_ID_BYTES],
                       mg_comm** out);
mg_status mg_comm_destroy(mg_comm* comm);
/* In-place sum of an f32 buffer across the group (replaces the serial reduce-to-root +
 * copy-back of src/multi/tensor_parallel.rs:697-734). */
mg_status mg_comm_all_reduce(mg_comm* comm, mg_buffer* buffer);
/* Failure handling.  The reference's peer copies have no failure path of their own; here
 * the communicator runs in NCCL's non-blocking mode and every NCCL call is bounded: the host
 * polls the call until it settles, and after the group's timeout (default 300 s, or
 * MAGNETAR_CUDA_COMM_TIMEOUT_MS, or mg_comm_set_timeout) the communicator is aborted and the
 * call fails with MG_DEVICE_UNAVAILABLE; an asynchronous NCCL error aborts it with
 * MG_DRIVER_FAILED.  An aborted communicator refuses all further work.
 * mg_comm_check polls once for an asynchronous error; mg_comm_wait waits, bounded, for the
 * group's enqueued work on this device (the compute and all-reduce streams) to finish and
 * aborts on timeout; mg_comm_abort aborts at once (a rank that learnt on the host that a peer
 * is gone). */
mg_status mg_comm_set_timeout(mg_comm* comm, int64_t timeout_ms);
mg_status mg_comm_check(mg_comm* comm);
mg_status mg_comm_wait(mg_comm* comm, int64_t timeout_ms);
mg_status mg_comm_abort(mg_comm* comm);
int mg_comm_is_aborted(const mg_comm* comm);

/* Measurement of mg_tp_mlp (no reference interface: the split the reference's tensor-parallel
 * MLP, src/multi/tensor_parallel.rs:697-734, leaves unmeasured).  With timing on, each
 * mg_tp_mlp call records three events on the compute stream: its start, the end of its last
 * down-projection chunk, and the join of the all-reduce stream.  mg_comm_mlp_timing waits for
 * the last timed call and returns start -> compute end (the gated and down GEMMs, with the
 * overlapped all-reduces running beside them) and compute end -> join (the all-reduce time
 * left exposed after the last GEMM).  MG_INVALID_ARGUMENT when no call was timed. */
mg_status mg_comm_set_mlp_timing(mg_comm* comm, int on);
mg_status mg_comm_mlp_timing(mg_comm* comm, float* compute_ms, float* exposed_ms);
/* Host-only test hook of the bounded settle: drives the poll loop with a scripted sequence of
 * NCCL results (0 success, 7 in progress, anything else an error; the last repeats) instead of
 * a communicator.  Returns the status the settle ends with; *aborted counts the aborts, *polls
 * the polls.  No GPU or NCCL call is made. */
mg_status mg_comm_settle_selftest(const int* states, int count, int64_t timeout_ms, int* aborted, int* polls);
/* The [start, end) share of `extent` that `member` of `parts` holds, aligned to 32 when
 * every part can hold at least one 32-block (src/multi/tensor_parallel.rs:82-86, 300-307). */
mg_status mg_tp_share(uint64_t extent, int parts, int member, uint64_t* start, uint64_t* end);
/* The tensor-parallel SwiGLU MLP of one rank: h = silu(x G_s) * (x U_s) on the rank's
 * column shards, y = h D_s on its row shard, then the sum over ranks, the all-reduce
 * chunked along tokens so that it overlaps the down projection. */
mg_status mg_tp_mlp(mg_comm* comm, const mg_buffer* x, const mg_buffer* gate_shard,
                    const mg_buffer* up_shard, const mg_buffer* down_shard, int chunks,
                    mg_buffer** out);
/* Executor-level plan (src/multi.rs:543-562): weight ids split by columns (kind 0) or
 * rows (kind 1) across the communicator's ranks; write_weight_tensor then keeps this
 * rank's share, and invocations reading a row-split weight are all-reduced. */
mg_status mg_executor_attach_comm(mg_executor* ex, mg_comm* comm);
mg_status mg_executor_apply_tensor_parallel(mg_executor* ex, int count, const char* const* weight_ids,
                                            const int* kinds);

#ifdef __cplusplus
}
#endif

#endif /* MAGNETAR_CUDA_H */
