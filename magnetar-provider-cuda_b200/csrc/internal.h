// Internal declarations shared by the provider's translation units: device and buffer
// objects behind the C ABI, the status/error plumbing, and the launch functions of every
// kernel.  Nothing here is part of the ABI.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdarg>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <utility>
#include <vector>

#include "../../include/magnetar_cuda.h"

namespace mg {

// ---- errors --------------------------------------------------------------------------
// Sets the calling thread's last-error detail and returns `status`.
mg_status fail(mg_status status, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
// Maps a CUDA runtime error to the reference's categories (src/error.rs:71-91).
mg_status from_cuda(cudaError_t err, const char* what);
void clear_error();

#define MG_TRY(expr)                          \
    do {                                      \
        mg_status _s = (expr);                \
        if (_s != MG_OK) return _s;           \
    } while (0)

#define MG_CUDA(expr, what)                              \
    do {                                                 \
        cudaError_t _e = (expr);                         \
        if (_e != cudaSuccess) return mg::from_cuda(_e, what); \
    } while (0)

// ---- device ----------------------------------------------------------------------------
struct Device {
    int ordinal = 0;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;  // where work is enqueued
    cudaMemPool_t pool = nullptr;
    int sm_count = 148;
    int sm_major = 10, sm_minor = 0;
    std::atomic<uint64_t> uploads{0}, downloads{0}, launches{0};
    // The open handle, every live buffer and every communicator hold a reference; the device's
    // stream, pool and status words go when the last is dropped, so a buffer released after
    // mg_device_close still frees into a live pool.  A closed device refuses new work.
    std::atomic<int> refs{1};
    std::atomic<bool> closed{false};
    // Device-side words (128 bytes): ints [0] invalid embedding id, [1] non-finite softmax row,
    // [2] kernel wait timeout, [3] a weight's lo term / compact check; bytes 32..39 the step
    // offset; 64..87 greedy selection's running max, ticket and result.  Pinned host mirror
    // (64 bytes) for the read backs.
    int* flags = nullptr;
    int* host_flags = nullptr;
    // The offset a captured step's advancing attributes add, read by its kernels at run time
    // (written before each replay).
    uint64_t* step_offset = nullptr;
    // Arrival counters of kernels whose last CTA finishes a tile (65,536 entries, zero
    // between kernels: the finishing CTA resets its entry).
    unsigned int* counters = nullptr;
    bool capturing = false;
    // Programmatic dependent launch between the provider's kernels (on unless the environment
    // sets MAGNETAR_CUDA_PDL=0).
    bool pdl = true;
    // Workspaces grown on demand (see scratch()); freed in stream order.
    void* scratch_ptr[8] = {nullptr};
    size_t scratch_bytes[8] = {0};
    // Allocations made while a step capture records the stream use plain cudaMalloc (a
    // captured graph must keep addressing the same memory on every replay); frees requested
    // during a capture wait until the capture ends.
    std::set<void*> plain_allocs;
    std::vector<void*> deferred_frees;
    // Device blocks that live captured steps address, each with the number of such steps.  A
    // block freed while a step still addresses it (a scratch workspace that grew, a weight's
    // dropped operand form, a replaced tensor) is only parked in held_frees; it is freed when
    // the last step addressing it is released, so a replay never touches freed memory.
    std::map<void*, int> graph_refs;
    std::set<void*> held_frees;
    // While a step capture records: every device block its launches address.
    std::set<void*> capture_touched;
    // Bumped whenever a buffer's prepared or compact operand form is dropped: a captured step
    // re-checks the forms it reads only when this moved since the capture.
    std::atomic<uint64_t> prep_gen{0};
    // Guards the allocation bookkeeping above (several executors may share a device).
    std::mutex mem_lock;
};

// Frees the allocations deferred while a capture was recording.
void flush_deferred_frees(Device* d);

// Captured-step bookkeeping: graph_touch records a block the capture in progress addresses
// (no-op outside a capture); graph_take hands the recorded set to the step being made;
// graph_hold / graph_release count a step's blocks in and out (the last release frees what
// was freed meanwhile).
void graph_touch(Device* d, const void* ptr);
std::vector<void*> graph_take(Device* d);
void graph_hold(Device* d, const std::vector<void*>& blocks);
void graph_release(Device* d, const std::vector<void*>& blocks);

void device_ref(Device* d);
// Drops one reference; the last one destroys the device.
void device_unref(Device* d);

mg_status device_check(mg_device* d);
inline Device* dev(mg_device* d) { return reinterpret_cast<Device*>(d); }

// Stream-ordered allocation from the device pool.
mg_status device_alloc(Device* d, size_t bytes, void** ptr);
void device_free(Device* d, void* ptr);

// Scratch memory: a per-device growable workspace (stream-ordered, reused across calls).
mg_status scratch(Device* d, int slot, size_t bytes, void** ptr);

// ---- buffers -----------------------------------------------------------------------------
struct Buffer {
    Device* device = nullptr;
    mg_dtype dtype = MG_F32;
    int rank = 0;
    uint64_t shape[MG_MAX_RANK] = {0};
    void* ptr = nullptr;
    uint64_t count = 0;  // elements
    bool owned = true;
    // A weight keeps the tensor-core matmul's operand form of itself once a matmul has read
    // it: the K-major tf32 hi/lo terms ([n, kp] each, hi first), built on first use with the
    // transpose flag it was read with, and dropped whenever the buffer's contents change.
    bool is_weight = false;
    // Set when the buffer becomes a weight: the kernel just before the next matmul may have
    // written it, so that matmul reads it only after its dependency wait.  Cleared by that
    // matmul; later ones may start loading the weight before the wait.
    bool weight_fresh = false;
    float* prep = nullptr;
    uint64_t prep_n = 0, prep_k = 0, prep_kp = 0;
    int prep_transposed = -1;
    // Every lo term of the prepared form is zero: the weight's values are exactly tf32 (as every
    // bfloat16 checkpoint's are), and the tensor-core matmul reads and multiplies hi alone.
    bool prep_one_term = false;
    // A compact weight: a matrix of at least kCompactMinElements values, every one exactly a
    // bfloat16 value, also kept as its bfloat16 bits ([k, n] as stored), which the few-row matmul
    // streams instead of the f32 values -- half the bytes, the same results.  Built on the first
    // such matmul that reads the weight, dropped with the prepared form.  compact_state: 0 not yet
    // checked, 1 built, -1 some value is not exactly bfloat16.
    uint16_t* compact = nullptr;
    int compact_state = 0;
    // A packed Q8_0 weight (dtype MG_Q8_0): ptr holds the int8 quants in stored row-major order
    // ([q8_rows, q8_cols]), q8_scales one f32 per 32 of them; the logical matrix (shape, count) is
    // the stored one, or its transpose when q8_transposed.
    float* q8_scales = nullptr;
    uint64_t q8_rows = 0, q8_cols = 0;
    int q8_transposed = 0;
    // Tiled layout (transposed storage with q8_cols a multiple of 128, the few-row matmul's
    // operand): per 256 stored rows and 128 stored columns one contiguous 32 KB record of quants
    // (each row's 128 quants in eight 16-byte pieces, piece j at position j ^ (row % 8)) and one
    // 4 KB record of scales ([256][4]), records ordered tile-major; stored rows padded to a
    // multiple of 256 with zeros.  Otherwise quants [q8_rows][q8_cols] and scales one per 32.
    int q8_tiled = 0;
};

// Rows a packed weight's arrays hold (padded when tiled), and the arrays' bytes.
inline uint64_t q8_rows_held(const Buffer* b) { return b->q8_tiled ? (b->q8_rows + 255) / 256 * 256 : b->q8_rows; }
inline uint64_t q8_quant_bytes(const Buffer* b) { return q8_rows_held(b) * b->q8_cols; }
inline uint64_t q8_scale_bytes(const Buffer* b) { return q8_rows_held(b) * b->q8_cols / 32 * sizeof(float); }

// Weights smaller than this stay f32 only (src/kernels.rs:506-510).
constexpr uint64_t kCompactMinElements = 1ull << 16;

// Drops a weight's prepared operand form (its contents are about to change).
void buffer_drop_prep(Buffer* b);

inline Buffer* buf(mg_buffer* b) { return reinterpret_cast<Buffer*>(b); }
inline const Buffer* buf(const mg_buffer* b) { return reinterpret_cast<const Buffer*>(b); }
inline size_t dtype_size(mg_dtype t) { return t == MG_F32 ? 4 : t == MG_Q8_0 ? 1 : 2; }
const char* dtype_name(mg_dtype t);
std::string shape_str(const Buffer* b);
bool same_shape(const Buffer* a, const Buffer* b);

mg_status buffer_new(Device* d, mg_dtype dtype, int rank, const uint64_t* shape, Buffer** out);
void buffer_free(Buffer* b);
// Output-offer rule: reuse *out when it matches (dtype, element count), else allocate.
mg_status output_for(Device* d, mg_dtype dtype, int rank, const uint64_t* shape, mg_buffer** out,
                     Buffer** result);

// ---- launches (all enqueue on `stream`, return cudaGetLastError() mapped) ---------------
namespace k {
mg_status add(Device* d, const float* a, const float* b, float* out, uint64_t n);
mg_status bias_add(Device* d, const float* a, const float* bias, float* out, uint64_t cols, uint64_t n);
mg_status mul(Device* d, const float* a, const float* b, float* out, uint64_t n);
mg_status mul_scalar(Device* d, const float* a, const float* b, float* out, uint64_t n);
mg_status scale(Device* d, const float* x, float* out, float factor, uint64_t n);
mg_status silu(Device* d, const float* x, float* out, uint64_t n);
mg_status gelu_tanh(Device* d, const float* x, float* out, uint64_t n);
mg_status sigmoid(Device* d, const float* x, float* out, uint64_t n);
mg_status softcap(Device* d, const float* x, float* out, float cap, uint64_t n);
mg_status row_scale(Device* d, const float* x, const float* scale, float* out, uint64_t rows, uint64_t cols);
mg_status concat_heads(Device* d, const float* a, const float* b, float* out, uint64_t rows, uint64_t heads,
                       uint64_t a_width, uint64_t b_width, uint64_t b_heads);
mg_status batched_matmul(Device* d, const float* a, const float* b, float* out, uint64_t rows, uint64_t groups,
                         uint64_t k, uint64_t n, int transpose_b);
mg_status silu_mul(Device* d, const float* g, const float* u, float* out, uint64_t n);
mg_status half_binary(Device* d, const uint16_t* a, const uint16_t* b, uint16_t* out, uint64_t n,
                      mg_dtype dtype, int op);
mg_status half_binary_f32(Device* d, const float* a, const float* b, float* out, uint64_t n,
                          mg_dtype dtype, int op);
mg_status encode_half(Device* d, const float* in, uint16_t* out, uint64_t n, mg_dtype dtype);
mg_status decode_half(Device* d, const uint16_t* in, float* out, uint64_t n, mg_dtype dtype);
mg_status fill_zero(Device* d, void* ptr, uint64_t bytes);
struct KvWriteArgs {
    const float* rows;
    float* store;
    uint64_t count, width, row_offset, capacity;
    const uint64_t* step;  // a captured step's advancing row offset (null: none)
};
mg_status kv_write(Device* d, const KvWriteArgs& a);
// *dst = value, in stream order (a captured step's offset before its replay).
mg_status set_step_offset(Device* d, uint64_t* dst, uint64_t value);

// The largest greedy-selection key of a logits row (0: no column eligible); `excluded` holds
// `count` host [start, end) pairs.  Reads the key back (synchronises the stream).
mg_status greedy_select(Device* d, const float* row, uint64_t cols, const uint64_t* excluded, uint32_t count,
                        float temperature, uint64_t* key);
mg_status embedding(Device* d, const float* table, const float* ids, float* out, uint64_t dim,
                    uint64_t num_ids, uint64_t vocab, int* flag, int has_scale, float scale);
mg_status rmsnorm(Device* d, const float* x, const float* w, float* out, uint64_t rows,
                  uint64_t cols, uint64_t w_stride, float eps);
struct EmbedArgs {
    const Buffer* packed = nullptr;  // a packed Q8_0 table (table then unused)
    const float* table;
    const float* ids;
    float* out;
    uint64_t dim, num_ids, vocab;
    int has_scale;
    float scale;
};
struct RmsArgs {
    const float* x;
    const float* w;  // null: no gain
    float* out;
    uint64_t rows, cols, w_stride;
    float eps;
};
// An embedding followed by an rmsnorm of its rows in one launch (the step capture's fusion):
// x = the gathered rows, out = rmsnorm(x), each exactly as the two kernels compute them.
// The lookup of a planned embedding: the f32 table's kernel or the packed table's.
mg_status embedding_run(Device* d, const EmbedArgs& e, int* flag);
bool embedding_rmsnorm_eligible(const EmbedArgs& e, const RmsArgs& r);
mg_status embedding_rmsnorm(Device* d, const EmbedArgs& e, const RmsArgs& r, int* flag);
struct RopeArgs {
    uint64_t rows, cols, half, dimension, position_offset, head_count, rotated_pairs;
    float base, scale, banded_factor, low_freq_factor, high_freq_factor, original_context_length;
    float yarn_factor, yarn_low, yarn_high, amplitude;
    int half_split;
    const uint64_t* step = nullptr;  // a captured step's advancing position offset (null: none)
};
mg_status rope(Device* d, const float* x, float* out, const RopeArgs& a);
mg_status softmax(Device* d, const float* x, float* out, uint64_t rows, uint64_t cols, int* flag);

// matmul family.  lda/ldb describe row-major storage; transposes select the index order.
struct GemmArgs {
    const float* a;
    const float* b;   // or gate
    const float* b2;  // up (gated) or nullptr
    float* out;
    const float* addend;
    int addend_mode;  // 0 none, 1 row [n], 2 full [m, n]
    uint64_t m, n, k;
    int transpose_a, transpose_b;
    int gated;
    // Prepared tensor-core forms of b / b2 (K-major tf32 hi, lo: [n, kp]); null = split per call.
    const float* b_prep[2];
    // The prepared forms existed before this call: no kernel earlier in the stream writes
    // them, so the GEMM may start loading them before it waits on its predecessor.
    int b_stable;
    // The prepared form's lo term is all zero (b / b2's values are exactly tf32).
    int b_one_term[2];
    // Compact (bfloat16-bit) forms of b / b2 for the few-row path; null = read the f32 values.
    const uint16_t* b16[2];
    // Packed Q8_0 b / b2 (b / b2 then unused); null for f32 operands.
    const Buffer* packed[2];
};
mg_status gemm(Device* d, const GemmArgs& g);
// Q8_0 packed weights: the 34-byte blocks split into quants and f32 scales; the logical matrix
// (or, stored_order, the stored one) dequantized; embedding rows of a packed table; the matmul
// with packed B (the few-row kernel, else dequantized for the call).
mg_status q8_unpack(Device* d, const uint8_t* blocks, const Buffer* b);
mg_status q8_dequantize(Device* d, const Buffer* b, float* out, bool stored_order);
mg_status q8_embedding(Device* d, const Buffer* table, const float* ids, float* out, uint64_t num_ids, int* flag,
                       int has_scale, float scale);
mg_status q8_matmul(Device* d, const GemmArgs& g);
// Writes the bfloat16 bits of b's `count` values to dst; sets *not_exact (a device word) when
// some value is not exactly a bfloat16 value.
mg_status gemv_compact_b(Device* d, const float* b, uint16_t* dst, uint64_t count, int* not_exact);
// Round-up of k the tensor-core path stores operands with.
inline uint64_t gemm_kp(uint64_t k) { return (k + 3) & ~3ull; }
// Fills dst ([n, kp] hi then [n, kp] lo) with the K-major tf32 terms of B ([k, n] row-major,
// or [n, k] when transposed).
// `lo_nonzero` (optional device word): set when any lo term is nonzero.
mg_status gemm_prepare_b(Device* d, const float* b, uint64_t k, uint64_t n, int transposed, float* dst,
                         int* lo_nonzero = nullptr);
// Whether the few-row (M <= 16) path takes a matmul.
bool gemv_eligible(const GemmArgs& g);
// Whether a matmul of these dimensions takes the tensor-core path (and so reads a prepared B).
bool gemm_uses_tensor_cores(uint64_t m, uint64_t n, uint64_t k, int transpose_b, const float* b);

struct AttentionArgs {
    const float* q;
    const float* k;
    const float* v;
    float* out;
    uint64_t seq_len, kv_seq_len, head_count, kv_head_count, head_dim, value_dim;
    uint64_t q_model_dim, kv_model_dim, v_model_dim;
    int causal;
    int64_t window;  // -1 none
    uint64_t query_position_offset;
    float scale;
    // A captured step's advancing key count (null: none): kv_seq_len + *step keys are admitted
    // at run time, at most kv_rows (the rows K and V hold).  Single query rows only.
    const uint64_t* step = nullptr;
    uint64_t kv_rows = 0;
};
mg_status attention(Device* d, const AttentionArgs& a);

// One launch for `count` (1-3) plain matmuls that share A and their shape (a grouped
// projection), each optionally also written rotated by `rope` into rope_outs[i] (null: none).
bool gemm_group_eligible(const GemmArgs* gs, int count, const RopeArgs* rope, float* const* rope_outs);
mg_status gemm_group(Device* d, const GemmArgs* gs, int count, const RopeArgs* rope, float* const* rope_outs);
}  // namespace k

// Everything a matmul / rope call does but the launch: validation, the output (offer rule) and
// the weights' operand forms.  The executor's step capture defers launches to fuse them; the
// launch is then k::gemm / k::gemm_group / k::rope with the result.
mg_status matmul_plan(mg_device* h, const mg_buffer* a, const mg_buffer* b, const mg_buffer* b2, const mg_buffer* addend,
                      int addend_mode, int ta, int tb, mg_buffer** out, k::GemmArgs* g);
mg_status rope_plan(mg_device* h, const mg_buffer* x, const mg_rope_params* p, mg_buffer** out, k::RopeArgs* a);
// The same for an embedding lookup and an rmsnorm (launch: k::embedding / k::rmsnorm, or the
// two fused by k::embedding_rmsnorm).
mg_status embedding_plan(mg_device* h, const mg_buffer* table, const mg_buffer* ids, int has_scale, float scale,
                         mg_buffer** out, k::EmbedArgs* e);
mg_status rmsnorm_plan(mg_device* h, const mg_buffer* x, const mg_buffer* w, float epsilon, uint64_t head_count,
                       uint64_t head_dimension, mg_buffer** out, k::RmsArgs* r);
// kv-write's validation (the write lands in `store` itself).
mg_status kv_write_plan(mg_device* h, mg_buffer* store, const mg_buffer* rows, uint64_t row_offset, k::KvWriteArgs* a);
// attention's validation and output (launch: k::attention).
mg_status attention_plan(mg_device* h, const mg_buffer* q, const mg_buffer* k, const mg_buffer* v,
                         const mg_attention_params* p, mg_buffer** out, k::AttentionArgs* a);

inline mg_status launched(Device* d, const char* what) {
    d->launches.fetch_add(1, std::memory_order_relaxed);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return from_cuda(e, what);
    return MG_OK;
}

// ---- programmatic dependent launch --------------------------------------------------------
// A chain of small kernels (a decoder layer) spends much of its time between kernels: the
// next grid is scheduled only after the previous one has drained.  Kernels launched through
// enqueue() may instead be scheduled while the previous kernel of the stream still runs; each
// of them starts with pdl_enter(), which waits until the kernels it depends on have completed
// and their memory is visible, and only then lets the next kernel of the stream be scheduled.
// Before pdl_enter() a kernel reads no global memory that an earlier kernel may write (a
// prepared weight is the one exception taken), writes none, and may allocate tensor memory
// only if every kernel using tensor memory does so before its own pdl_enter(): the next grid
// is scheduled only after every CTA of this one has passed pdl_enter(), so each CTA that
// waits for tensor memory waits on a grid that is already running and never on its successor.
// Kernels launched without the attribute pass pdl_enter() at once.
#ifdef __CUDACC__
__device__ __forceinline__ void pdl_enter() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
#endif

// Enqueues `kernel` on the device stream (a launch failure is left for launched() to read).
template <typename... KArgs, typename... Args>
inline void enqueue(Device* d, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = d->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = d->pdl ? 1 : 0;
    (void)cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace mg
