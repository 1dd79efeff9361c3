// C ABI of the kernel entry points: each validates its operands exactly as the matching
// `CudaKernels` method of the reference does (shape errors -> ShapeUnsupported, non-f32 ->
// DTypeUnsupported), picks the output buffer by the output-offer rule, and enqueues the
// kernel.  Citations are to src/kernels.rs of astorise/Magnetar-provider-CUDA.
#include <cmath>
#include <cstring>

#include "internal.h"

using namespace mg;

namespace {

mg_status need(const mg_buffer* b, const char* what) {
    if (!b) return fail(MG_INVALID_ARGUMENT, "null %s buffer", what);
    return MG_OK;
}

// Kernels read f32 operands only (src/kernels.rs:1375-1383).
mg_status require_f32(const Buffer* b, const char* what) {
    if (b->dtype != MG_F32)
        return fail(MG_DTYPE_UNSUPPORTED, "%s does not read %s operands", what, dtype_name(b->dtype));
    return MG_OK;
}

mg_status same_device(Device* d, const Buffer* b) {
    if (b->device != d) return fail(MG_INVALID_ARGUMENT, "buffer belongs to another device");
    return MG_OK;
}

// src/kernels.rs:7134-7142
mg_status rows_cols(const Buffer* b, uint64_t* rows, uint64_t* cols) {
    if (b->rank != 2) return fail(MG_SHAPE_UNSUPPORTED, "expected rank-2 tensor, got shape %s", shape_str(b).c_str());
    *rows = b->shape[0];
    *cols = b->shape[1];
    return MG_OK;
}

bool is_row(const Buffer* b, uint64_t n) {
    return (b->rank == 1 && b->shape[0] == n) || (b->rank == 2 && b->shape[0] == 1 && b->shape[1] == n);
}

// Waits for the stream and reads the device status words (the reference's flag reads).
mg_status read_flags(Device* d, int* host) {
    MG_CUDA(cudaMemcpyAsync(d->host_flags, d->flags, 4 * sizeof(int), cudaMemcpyDeviceToHost, d->stream), "reading a status flag");
    MG_CUDA(cudaStreamSynchronize(d->stream), "waiting for the device");
    memcpy(host, d->host_flags, 4 * sizeof(int));
    d->downloads.fetch_add(1);
    return MG_OK;
}

// add with same-shape or row broadcast (src/kernels.rs:2956-3015)
mg_status add_impl(mg_device* h, const mg_buffer* ah, const mg_buffer* bh, mg_buffer** out, const char* what) {
    MG_TRY(device_check(h));
    MG_TRY(need(ah, "a"));
    MG_TRY(need(bh, "b"));
    Device* d = dev(h);
    const Buffer* a = buf(ah);
    const Buffer* b = buf(bh);
    MG_TRY(same_device(d, a));
    MG_TRY(same_device(d, b));
    MG_TRY(require_f32(a, what));
    MG_TRY(require_f32(b, what));
    if (same_shape(a, b)) {
        Buffer* o;
        MG_TRY(output_for(d, MG_F32, a->rank, a->shape, out, &o));
        return k::add(d, (const float*)a->ptr, (const float*)b->ptr, (float*)o->ptr, a->count);
    }
    if (a->rank == 0) return fail(MG_SHAPE_UNSUPPORTED, "add expects at least one dimension");
    const uint64_t cols = a->shape[a->rank - 1];
    if (!is_row(b, cols))
        return fail(MG_SHAPE_UNSUPPORTED, "add expects b to match a's shape %s or broadcast as [%llu]/[1, %llu], got %s",
                    shape_str(a).c_str(), (unsigned long long)cols, (unsigned long long)cols, shape_str(b).c_str());
    if (cols == 0 || a->count % cols != 0)
        return fail(MG_SHAPE_UNSUPPORTED, "add data length %llu is not divisible by broadcast dimension %llu",
                    (unsigned long long)a->count, (unsigned long long)cols);
    Buffer* o;
    MG_TRY(output_for(d, MG_F32, a->rank, a->shape, out, &o));
    return k::bias_add(d, (const float*)a->ptr, (const float*)b->ptr, (float*)o->ptr, cols, a->count);
}

mg_status unary_prep(mg_device* h, const mg_buffer* xh, mg_buffer** out, const char* what, Device** d, const Buffer** x,
                     Buffer** o) {
    MG_TRY(device_check(h));
    MG_TRY(need(xh, "input"));
    *d = dev(h);
    *x = buf(xh);
    MG_TRY(same_device(*d, *x));
    MG_TRY(require_f32(*x, what));
    return output_for(*d, MG_F32, (*x)->rank, (*x)->shape, out, o);
}

mg_status half_impl(mg_device* h, const mg_buffer* ah, const mg_buffer* bh, mg_buffer** out, int op) {
    MG_TRY(device_check(h));
    MG_TRY(need(ah, "a"));
    MG_TRY(need(bh, "b"));
    Device* d = dev(h);
    const Buffer* a = buf(ah);
    const Buffer* b = buf(bh);
    MG_TRY(same_device(d, a));
    MG_TRY(same_device(d, b));
    // src/kernels.rs:2227-2266: both operands share shape and half dtype.
    if (a->dtype == MG_F32 || b->dtype == MG_F32)
        return fail(MG_DTYPE_UNSUPPORTED, "%s expects f16 or bf16 operands", op ? "mul-half" : "add-half");
    if (a->dtype != b->dtype)
        return fail(MG_DTYPE_UNSUPPORTED, "%s operands differ in dtype: %s vs %s", op ? "mul-half" : "add-half",
                    dtype_name(a->dtype), dtype_name(b->dtype));
    if (!same_shape(a, b))
        return fail(MG_SHAPE_UNSUPPORTED, "shape mismatch: %s vs %s", shape_str(a).c_str(), shape_str(b).c_str());
    Buffer* o;
    MG_TRY(output_for(d, a->dtype, a->rank, a->shape, out, &o));
    return k::half_binary(d, (const uint16_t*)a->ptr, (const uint16_t*)b->ptr, (uint16_t*)o->ptr, a->count, a->dtype, op);
}

enum AddendMode { kNone = 0, kRow = 1, kFull = 2 };

// The prepared tensor-core operand form of a weight read as matmul B, built on first use.
mg_status weight_prep(Device* d, const Buffer* cb, uint64_t k, uint64_t n, int transposed, const float** out,
                      bool* built, int* one_term) {
    *out = nullptr;
    *one_term = 0;
    if (!cb || !cb->is_weight) return MG_OK;
    Buffer* b = const_cast<Buffer*>(cb);  // the prepared form is a cache of the buffer's contents
    if (b->prep && b->prep_n == n && b->prep_k == k && b->prep_transposed == transposed) {
        *out = b->prep;
        *one_term = b->prep_one_term ? 1 : 0;
        return MG_OK;
    }
    *built = true;
    buffer_drop_prep(b);
    const uint64_t kp = k::gemm_kp(k);
    void* mem = nullptr;
    MG_TRY(device_alloc(d, 2 * n * kp * sizeof(float), &mem));
    // Whether the lo term is all zero is read back once, here (never while a capture records:
    // such a weight keeps both terms).
    int* lo_flag = d->capturing ? nullptr : d->flags + 3;
    if (lo_flag) MG_CUDA(cudaMemsetAsync(lo_flag, 0, sizeof(int), d->stream), "resetting the lo flag");
    mg_status s = k::gemm_prepare_b(d, (const float*)b->ptr, k, n, transposed, (float*)mem, lo_flag);
    int flags[4] = {0, 0, 0, 1};
    if (s == MG_OK && lo_flag) s = read_flags(d, flags);
    if (s != MG_OK) {
        device_free(d, mem);
        return s;
    }
    b->prep_one_term = flags[3] == 0;
    b->prep = (float*)mem;
    b->prep_n = n;
    b->prep_k = k;
    b->prep_kp = kp;
    b->prep_transposed = transposed;
    *out = b->prep;
    *one_term = b->prep_one_term ? 1 : 0;
    return MG_OK;
}

// The compact form of a weight read as the few-row matmul's B (src/kernels.rs:1668-1712: a
// matrix of at least 65536 values, all exactly bfloat16, is kept as bfloat16 bits): built and
// checked on first use -- one read-back, never while a capture records -- then reused until
// the weight's contents change.  Null when the weight is not compact.
mg_status weight_compact(Device* d, const Buffer* cb, uint64_t k, uint64_t n, const uint16_t** out) {
    *out = nullptr;
    Buffer* b = const_cast<Buffer*>(cb);  // the compact form is a cache of the buffer's contents
    if (!b->is_weight || b->rank != 2 || b->count < kCompactMinElements || b->count != k * n || n % 8 != 0) return MG_OK;
    if (b->compact_state == 1) {
        *out = b->compact;
        return MG_OK;
    }
    if (b->compact_state < 0 || d->capturing) return MG_OK;
    void* mem = nullptr;
    MG_TRY(device_alloc(d, b->count * sizeof(uint16_t), &mem));
    int* flag = d->flags + 3;
    const cudaError_t e = cudaMemsetAsync(flag, 0, sizeof(int), d->stream);
    mg_status s = e == cudaSuccess ? MG_OK : from_cuda(e, "resetting the compact flag");
    if (s == MG_OK) s = k::gemv_compact_b(d, (const float*)b->ptr, (uint16_t*)mem, b->count, flag);
    int flags[4] = {0, 0, 0, 1};
    if (s == MG_OK) s = read_flags(d, flags);
    if (s != MG_OK || flags[3] != 0) {
        device_free(d, mem);
        if (s == MG_OK) b->compact_state = -1;
        return s;
    }
    b->compact = (uint16_t*)mem;
    b->compact_state = 1;
    *out = b->compact;
    return MG_OK;
}

}  // namespace

namespace mg {
// src/kernels.rs:5518-5580: shapes, transposes and the addend's shape; the output and the
// weights' operand forms -- everything a matmul does but the launch.
mg_status matmul_plan(mg_device* h, const mg_buffer* ah, const mg_buffer* bh, const mg_buffer* b2h,
                      const mg_buffer* addh, int addend_mode, int ta, int tb, mg_buffer** out, k::GemmArgs* gp) {
    MG_TRY(device_check(h));
    MG_TRY(need(ah, "a"));
    MG_TRY(need(bh, "b"));
    Device* d = dev(h);
    const Buffer* a = buf(ah);
    const Buffer* b = buf(bh);
    MG_TRY(same_device(d, a));
    MG_TRY(same_device(d, b));
    uint64_t ar, ac, br, bc;
    MG_TRY(rows_cols(a, &ar, &ac));
    MG_TRY(rows_cols(b, &br, &bc));
    const uint64_t m = ta ? ac : ar, kk = ta ? ar : ac;
    const uint64_t k2 = tb ? bc : br, n = tb ? br : bc;
    if (kk != k2)
        return fail(MG_SHAPE_UNSUPPORTED, "matmul inner dimension mismatch: %llu vs %llu", (unsigned long long)kk,
                    (unsigned long long)k2);
    const Buffer* b2 = nullptr;
    if (b2h) {
        b2 = buf(b2h);
        MG_TRY(same_device(d, b2));
        if (!same_shape(b, b2))
            return fail(MG_SHAPE_UNSUPPORTED, "gated-matmul expects gate and up to share a shape, got %s and %s",
                        shape_str(b).c_str(), shape_str(b2).c_str());
        if (b2->dtype != MG_Q8_0) MG_TRY(require_f32(b2, "gated-matmul's up"));
    }
    const Buffer* add = nullptr;
    if (addh) {
        add = buf(addh);
        MG_TRY(same_device(d, add));
        if (addend_mode == kRow && !is_row(add, n))
            return fail(MG_SHAPE_UNSUPPORTED, "matmul-bias bias shape must be [%llu] or [1, %llu], got %s",
                        (unsigned long long)n, (unsigned long long)n, shape_str(add).c_str());
        if (addend_mode == kFull && !(add->rank == 2 && add->shape[0] == m && add->shape[1] == n))
            return fail(MG_SHAPE_UNSUPPORTED, "matmul-residual residual shape must be [%llu, %llu], got %s",
                        (unsigned long long)m, (unsigned long long)n, shape_str(add).c_str());
    }
    MG_TRY(require_f32(a, "matmul's a"));
    if (b->dtype != MG_Q8_0) MG_TRY(require_f32(b, "matmul's b"));
    if (add) MG_TRY(require_f32(add, "a fused matmul's addend"));
    const uint64_t shape[2] = {m, n};
    Buffer* o;
    MG_TRY(output_for(d, MG_F32, 2, shape, out, &o));
    k::GemmArgs g{};
    g.a = (const float*)a->ptr;
    g.b = (const float*)b->ptr;
    g.b2 = b2 ? (const float*)b2->ptr : nullptr;
    g.out = (float*)o->ptr;
    g.addend = add ? (const float*)add->ptr : nullptr;
    g.addend_mode = add ? addend_mode : kNone;
    g.m = m;
    g.n = n;
    g.k = kk;
    g.transpose_a = ta;
    g.transpose_b = tb;
    g.gated = b2 ? 1 : 0;
    g.b_prep[0] = g.b_prep[1] = nullptr;
    g.b16[0] = g.b16[1] = nullptr;
    g.packed[0] = b->dtype == MG_Q8_0 ? b : nullptr;
    g.packed[1] = b2 && b2->dtype == MG_Q8_0 ? b2 : nullptr;
    if (g.packed[0] || g.packed[1]) {
        // packed weights: read by the packed paths (src/kernels.rs:5581-5600)
        g.b_stable = 0;
    } else if (k::gemm_uses_tensor_cores(m, n, kk, tb, g.b)) {
        bool built = false;
        MG_TRY(weight_prep(d, b, kk, n, tb, &g.b_prep[0], &built, &g.b_one_term[0]));
        if (b2) MG_TRY(weight_prep(d, b2, kk, n, tb, &g.b_prep[1], &built, &g.b_one_term[1]));
        g.b_stable = !built && g.b_prep[0] && (!b2 || g.b_prep[1]);
    } else {
        // The GEMV path reads B as it is: before its dependency wait when B is a weight that
        // the preceding kernel cannot have written.
        auto settled = [](const Buffer* w) { return w->is_weight && !w->weight_fresh; };
        g.b_stable = settled(b) && (!b2 || settled(b2));
        if (k::gemv_eligible(g)) {
            MG_TRY(weight_compact(d, b, kk, n, &g.b16[0]));
            if (b2) MG_TRY(weight_compact(d, b2, kk, n, &g.b16[1]));
        }
        const_cast<Buffer*>(b)->weight_fresh = false;
        if (b2) const_cast<Buffer*>(b2)->weight_fresh = false;
    }
    *gp = g;
    return MG_OK;
}
}  // namespace mg

namespace {

mg_status matmul_impl(mg_device* h, const mg_buffer* ah, const mg_buffer* bh, const mg_buffer* b2h,
                      const mg_buffer* addh, int addend_mode, int ta, int tb, mg_buffer** out) {
    k::GemmArgs g;
    MG_TRY(matmul_plan(h, ah, bh, b2h, addh, addend_mode, ta, tb, out, &g));
    return k::gemm(dev(h), g);
}

}  // namespace

extern "C" {

mg_status mg_add(mg_device* h, const mg_buffer* a, const mg_buffer* b, mg_buffer** out) {
    return add_impl(h, a, b, out, "add");
}

// src/kernels.rs:3039-3046
mg_status mg_residual_add(mg_device* h, const mg_buffer* input, const mg_buffer* residual, mg_buffer** out) {
    return add_impl(h, input, residual, out, "residual-add");
}

// src/kernels.rs:3017-3037; a [1] second operand scales every element (src/executor.rs:1917-1927)
mg_status mg_mul(mg_device* h, const mg_buffer* ah, const mg_buffer* bh, mg_buffer** out) {
    MG_TRY(device_check(h));
    MG_TRY(need(ah, "a"));
    MG_TRY(need(bh, "b"));
    Device* d = dev(h);
    const Buffer* a = buf(ah);
    const Buffer* b = buf(bh);
    MG_TRY(same_device(d, a));
    MG_TRY(same_device(d, b));
    MG_TRY(require_f32(a, "mul"));
    MG_TRY(require_f32(b, "mul"));
    const bool scalar = b->rank == 1 && b->shape[0] == 1 && !same_shape(a, b);
    if (!scalar && !same_shape(a, b))
        return fail(MG_SHAPE_UNSUPPORTED, "shape mismatch: %s vs %s", shape_str(a).c_str(), shape_str(b).c_str());
    Buffer* o;
    MG_TRY(output_for(d, MG_F32, a->rank, a->shape, out, &o));
    if (scalar) return k::mul_scalar(d, (const float*)a->ptr, (const float*)b->ptr, (float*)o->ptr, a->count);
    return k::mul(d, (const float*)a->ptr, (const float*)b->ptr, (float*)o->ptr, a->count);
}

mg_status mg_scale(mg_device* h, const mg_buffer* xh, float factor, mg_buffer** out) {
    Device* d;
    const Buffer* x;
    Buffer* o;
    MG_TRY(unary_prep(h, xh, out, "scale", &d, &x, &o));
    return k::scale(d, (const float*)x->ptr, (float*)o->ptr, factor, x->count);
}

mg_status mg_silu(mg_device* h, const mg_buffer* xh, mg_buffer** out) {
    Device* d;
    const Buffer* x;
    Buffer* o;
    MG_TRY(unary_prep(h, xh, out, "silu", &d, &x, &o));
    return k::silu(d, (const float*)x->ptr, (float*)o->ptr, x->count);
}

// src/kernels.rs:3167-3170 (the tanh approximation)
mg_status mg_gelu_tanh(mg_device* h, const mg_buffer* xh, mg_buffer** out) {
    Device* d;
    const Buffer* x;
    Buffer* o;
    MG_TRY(unary_prep(h, xh, out, "gelu", &d, &x, &o));
    return k::gelu_tanh(d, (const float*)x->ptr, (float*)o->ptr, x->count);
}

// src/kernels.rs:3121-3125
mg_status mg_sigmoid(mg_device* h, const mg_buffer* xh, mg_buffer** out) {
    Device* d;
    const Buffer* x;
    Buffer* o;
    MG_TRY(unary_prep(h, xh, out, "sigmoid", &d, &x, &o));
    return k::sigmoid(d, (const float*)x->ptr, (float*)o->ptr, x->count);
}

// src/kernels.rs:3211-3224
mg_status mg_softcap(mg_device* h, const mg_buffer* xh, float cap, mg_buffer** out) {
    if (!std::isfinite(cap) || !(cap > 0.0f))
        return fail(MG_SHAPE_UNSUPPORTED, "softcap cap %g must be finite and positive", (double)cap);
    Device* d;
    const Buffer* x;
    Buffer* o;
    MG_TRY(unary_prep(h, xh, out, "softcap", &d, &x, &o));
    return k::softcap(d, (const float*)x->ptr, (float*)o->ptr, cap, x->count);
}

// src/kernels.rs:3255-3290: out[t, :] = x[t, :] * scale[t], scale of [T, 1] or [T]
mg_status mg_row_scale(mg_device* h, const mg_buffer* xh, const mg_buffer* sh, mg_buffer** out) {
    MG_TRY(device_check(h));
    MG_TRY(need(xh, "input"));
    MG_TRY(need(sh, "scale"));
    Device* d = dev(h);
    const Buffer* x = buf(xh);
    const Buffer* sc = buf(sh);
    MG_TRY(same_device(d, x));
    MG_TRY(same_device(d, sc));
    MG_TRY(require_f32(x, "row-scale"));
    MG_TRY(require_f32(sc, "row-scale"));
    uint64_t rows, cols;
    MG_TRY(rows_cols(x, &rows, &cols));
    if (sc->count != rows)
        return fail(MG_SHAPE_UNSUPPORTED, "row-scale expects one scale per row of %s, got %s", shape_str(x).c_str(),
                    shape_str(sc).c_str());
    Buffer* o;
    MG_TRY(output_for(d, MG_F32, x->rank, x->shape, out, &o));
    return k::row_scale(d, (const float*)x->ptr, (const float*)sc->ptr, (float*)o->ptr, rows, cols);
}

// src/kernels.rs:3058-3100: along the first dimension (the trailing ones must agree)
mg_status mg_concat(mg_device* h, const mg_buffer* ah, const mg_buffer* bh, mg_buffer** out) {
    MG_TRY(device_check(h));
    MG_TRY(need(ah, "a"));
    MG_TRY(need(bh, "b"));
    Device* d = dev(h);
    const Buffer* a = buf(ah);
    const Buffer* b = buf(bh);
    MG_TRY(same_device(d, a));
    MG_TRY(same_device(d, b));
    MG_TRY(require_f32(a, "concat"));
    MG_TRY(require_f32(b, "concat"));
    if (a->rank == 0) return fail(MG_SHAPE_UNSUPPORTED, "concat expects a to have at least one dimension");
    if (b->rank == 0) return fail(MG_SHAPE_UNSUPPORTED, "concat expects b to have at least one dimension");
    bool same_rest = a->rank == b->rank;
    for (int i = 1; same_rest && i < a->rank; i++) same_rest = a->shape[i] == b->shape[i];
    if (!same_rest)
        return fail(MG_SHAPE_UNSUPPORTED, "concat expects a and b to share trailing dimensions, got %s and %s",
                    shape_str(a).c_str(), shape_str(b).c_str());
    uint64_t shape[MG_MAX_RANK];
    for (int i = 0; i < a->rank; i++) shape[i] = a->shape[i];
    shape[0] = a->shape[0] + b->shape[0];
    Buffer* o;
    MG_TRY(output_for(d, MG_F32, a->rank, shape, out, &o));
    if (a->count)
        MG_CUDA(cudaMemcpyAsync(o->ptr, a->ptr, a->count * 4, cudaMemcpyDeviceToDevice, d->stream), "concat copy");
    if (b->count)
        MG_CUDA(cudaMemcpyAsync((float*)o->ptr + a->count, b->ptr, b->count * 4, cudaMemcpyDeviceToDevice, d->stream),
                "concat copy");
    return MG_OK;
}

// src/kernels.rs:7084-7130: each output row holds head_count heads, head h being a's head h
// then b's head h (second_head_count == head_count) or b's only head (second_head_count == 1).
mg_status mg_concat_heads(mg_device* h, const mg_buffer* ah, const mg_buffer* bh, uint64_t head_count,
                          uint64_t second_head_count, mg_buffer** out) {
    MG_TRY(device_check(h));
    MG_TRY(need(ah, "a"));
    MG_TRY(need(bh, "b"));
    Device* d = dev(h);
    const Buffer* a = buf(ah);
    const Buffer* b = buf(bh);
    MG_TRY(same_device(d, a));
    MG_TRY(same_device(d, b));
    MG_TRY(require_f32(a, "concat"));
    MG_TRY(require_f32(b, "concat"));
    uint64_t rows, a_cols, b_rows, b_cols;
    MG_TRY(rows_cols(a, &rows, &a_cols));
    MG_TRY(rows_cols(b, &b_rows, &b_cols));
    if (rows != b_rows)
        return fail(MG_SHAPE_UNSUPPORTED, "concat across heads needs inputs with the same rows, got %s and %s",
                    shape_str(a).c_str(), shape_str(b).c_str());
    if (head_count == 0 || a_cols % head_count != 0 || second_head_count == 0 ||
        (second_head_count != 1 && second_head_count != head_count) || b_cols % second_head_count != 0)
        return fail(MG_SHAPE_UNSUPPORTED,
                    "concat across heads cannot split %s into %llu heads and %s into %llu (the second input has "
                    "one head or as many as the first)",
                    shape_str(a).c_str(), (unsigned long long)head_count, shape_str(b).c_str(),
                    (unsigned long long)second_head_count);
    const uint64_t a_width = a_cols / head_count, b_width = b_cols / second_head_count;
    const uint64_t shape[2] = {rows, head_count * (a_width + b_width)};
    Buffer* o;
    MG_TRY(output_for(d, MG_F32, 2, shape, out, &o));
    return k::concat_heads(d, (const float*)a->ptr, (const float*)b->ptr, (float*)o->ptr, rows, head_count, a_width,
                           b_width, second_head_count);
}

// src/kernels.rs:5882-5950
mg_status mg_batched_matmul(mg_device* h, const mg_buffer* ah, const mg_buffer* bh, uint64_t groups, int transpose_b,
                            mg_buffer** out) {
    MG_TRY(device_check(h));
    MG_TRY(need(ah, "a"));
    MG_TRY(need(bh, "b"));
    Device* d = dev(h);
    const Buffer* a = buf(ah);
    const Buffer* b = buf(bh);
    MG_TRY(same_device(d, a));
    MG_TRY(same_device(d, b));
    MG_TRY(require_f32(a, "batched-matmul"));
    MG_TRY(require_f32(b, "batched-matmul"));
    uint64_t rows, a_cols, b_rows, b_cols;
    MG_TRY(rows_cols(a, &rows, &a_cols));
    MG_TRY(rows_cols(b, &b_rows, &b_cols));
    const bool fits = groups > 0 && a_cols % groups == 0 && b_rows % groups == 0 &&
                      (transpose_b ? b_cols == a_cols / groups : b_rows == a_cols);
    if (!fits)
        return fail(MG_SHAPE_UNSUPPORTED, "batched-matmul of %llu groups (transpose_b %s) cannot take %s and %s",
                    (unsigned long long)groups, transpose_b ? "true" : "false", shape_str(a).c_str(),
                    shape_str(b).c_str());
    const uint64_t k = a_cols / groups, n = transpose_b ? b_rows / groups : b_cols;
    const uint64_t shape[2] = {rows, groups * n};
    Buffer* o;
    MG_TRY(output_for(d, MG_F32, 2, shape, out, &o));
    return k::batched_matmul(d, (const float*)a->ptr, (const float*)b->ptr, (float*)o->ptr, rows, groups, k, n,
                             transpose_b);
}

// src/kernels.rs:4492-4523
mg_status mg_silu_mul(mg_device* h, const mg_buffer* gh, const mg_buffer* uh, mg_buffer** out) {
    MG_TRY(device_check(h));
    MG_TRY(need(gh, "gate"));
    MG_TRY(need(uh, "up"));
    Device* d = dev(h);
    const Buffer* g = buf(gh);
    const Buffer* u = buf(uh);
    MG_TRY(same_device(d, g));
    MG_TRY(same_device(d, u));
    MG_TRY(require_f32(g, "silu-mul"));
    MG_TRY(require_f32(u, "silu-mul"));
    if (!same_shape(g, u))
        return fail(MG_SHAPE_UNSUPPORTED, "silu-mul expects gate and up to share a shape, got %s and %s",
                    shape_str(g).c_str(), shape_str(u).c_str());
    Buffer* o;
    MG_TRY(output_for(d, MG_F32, g->rank, g->shape, out, &o));
    return k::silu_mul(d, (const float*)g->ptr, (const float*)u->ptr, (float*)o->ptr, g->count);
}

mg_status mg_add_half(mg_device* h, const mg_buffer* a, const mg_buffer* b, mg_buffer** out) {
    return half_impl(h, a, b, out, 0);
}

mg_status mg_mul_half(mg_device* h, const mg_buffer* a, const mg_buffer* b, mg_buffer** out) {
    return half_impl(h, a, b, out, 1);
}

mg_status mg_half_binary_f32(mg_device* h, const mg_buffer* ah, const mg_buffer* bh, mg_dtype dtype, int op,
                             mg_buffer** out) {
    MG_TRY(device_check(h));
    MG_TRY(need(ah, "a"));
    MG_TRY(need(bh, "b"));
    Device* d = dev(h);
    const Buffer* a = buf(ah);
    const Buffer* b = buf(bh);
    MG_TRY(same_device(d, a));
    MG_TRY(same_device(d, b));
    if (dtype != MG_F16 && dtype != MG_BF16)
        return fail(MG_DTYPE_UNSUPPORTED, "add-half/mul-half need an f16 or bf16 descriptor, got %s", dtype_name(dtype));
    MG_TRY(require_f32(a, "an f32-resident half op"));
    MG_TRY(require_f32(b, "an f32-resident half op"));
    if (!same_shape(a, b))
        return fail(MG_SHAPE_UNSUPPORTED, "shape mismatch: %s vs %s", shape_str(a).c_str(), shape_str(b).c_str());
    Buffer* o;
    MG_TRY(output_for(d, MG_F32, a->rank, a->shape, out, &o));
    return k::half_binary_f32(d, (const float*)a->ptr, (const float*)b->ptr, (float*)o->ptr, a->count, dtype, op ? 1 : 0);
}

}  // extern "C"

namespace mg {
// src/kernels.rs:3833-3997 (f32 table path) and the executor's `scale` (src/executor.rs:1502-1518)
mg_status embedding_plan(mg_device* h, const mg_buffer* th, const mg_buffer* ih, int has_scale, float scale,
                         mg_buffer** out, k::EmbedArgs* e) {
    MG_TRY(device_check(h));
    MG_TRY(need(th, "table"));
    MG_TRY(need(ih, "ids"));
    Device* d = dev(h);
    const Buffer* t = buf(th);
    const Buffer* ids = buf(ih);
    MG_TRY(same_device(d, t));
    MG_TRY(same_device(d, ids));
    uint64_t vocab, dim;
    MG_TRY(rows_cols(t, &vocab, &dim));
    MG_TRY(require_f32(ids, "the embedding lookup's ids"));
    // a packed table is read row by row when stored untransposed (src/kernels.rs:1970-1982)
    if (t->dtype == MG_Q8_0 && t->q8_transposed)
        return fail(MG_DTYPE_UNSUPPORTED, "rows of a packed weight stored transposed");
    if (t->dtype != MG_Q8_0) MG_TRY(require_f32(t, "the embedding lookup's table"));
    const uint64_t shape[2] = {ids->count, dim};
    Buffer* o;
    MG_TRY(output_for(d, MG_F32, 2, shape, out, &o));
    e->packed = t->dtype == MG_Q8_0 ? t : nullptr;
    e->table = e->packed ? nullptr : (const float*)t->ptr;
    e->ids = (const float*)ids->ptr;
    e->out = (float*)o->ptr;
    e->dim = dim;
    e->num_ids = ids->count;
    e->vocab = vocab;
    e->has_scale = has_scale;
    e->scale = scale;
    return MG_OK;
}
}  // namespace mg

extern "C" {

mg_status mg_embedding(mg_device* h, const mg_buffer* th, const mg_buffer* ih, int has_scale, float scale,
                       mg_buffer** out) {
    k::EmbedArgs e;
    MG_TRY(embedding_plan(h, th, ih, has_scale, scale, out, &e));
    Device* d = dev(h);
    if (!d->capturing) MG_CUDA(cudaMemsetAsync(d->flags, 0, sizeof(int), d->stream), "resetting the id flag");
    MG_TRY(k::embedding_run(d, e, d->flags));
    if (d->capturing) return MG_OK;  // checked once the captured step has run
    int flags[4];
    MG_TRY(read_flags(d, flags));
    if (flags[0])
        return fail(MG_SHAPE_UNSUPPORTED, "embedding lookup id is not a valid in-range non-negative integer");
    return MG_OK;
}

}  // extern "C"

namespace mg {
// src/kernels.rs:4013-4104
mg_status rmsnorm_plan(mg_device* h, const mg_buffer* xh, const mg_buffer* wh, float epsilon, uint64_t head_count,
                       uint64_t head_dimension, mg_buffer** out, k::RmsArgs* r) {
    MG_TRY(device_check(h));
    MG_TRY(need(xh, "input"));
    Device* d = dev(h);
    const Buffer* x = buf(xh);
    MG_TRY(same_device(d, x));
    MG_TRY(require_f32(x, "rmsnorm"));
    const Buffer* w = wh ? buf(wh) : nullptr;
    if (w) {
        MG_TRY(same_device(d, w));
        MG_TRY(require_f32(w, "rmsnorm"));
    }
    if (x->rank == 0) return fail(MG_SHAPE_UNSUPPORTED, "RMSNorm expects at least one dimension");
    const uint64_t row_width = x->shape[x->rank - 1];
    const bool heads = head_count != 0 || head_dimension != 0;
    uint64_t cols = row_width;
    if (heads) {
        if (head_count == 0 || head_dimension == 0 || head_count * head_dimension != row_width ||
            row_width / head_count != head_dimension)
            return fail(MG_SHAPE_UNSUPPORTED, "RMSNorm's %llu heads of %llu do not tile rows of %llu",
                        (unsigned long long)head_count, (unsigned long long)head_dimension, (unsigned long long)row_width);
        cols = head_dimension;
    }
    if (cols == 0 || x->count % cols != 0)
        return fail(MG_SHAPE_UNSUPPORTED, "RMSNorm data length %llu is not divisible by hidden dimension %llu",
                    (unsigned long long)x->count, (unsigned long long)cols);
    const uint64_t rows = x->count / cols;
    uint64_t w_stride = 0;
    if (w) {
        if (is_row(w, cols)) {
            w_stride = 0;
        } else if (!heads && (same_shape(w, x) || (w->rank == 2 && w->shape[0] == rows && w->shape[1] == cols))) {
            w_stride = cols;
        } else {
            return fail(MG_SHAPE_UNSUPPORTED,
                        "RMSNorm weight shape must be [%llu], [1, %llu], input shape %s, or [%llu, %llu], got %s",
                        (unsigned long long)cols, (unsigned long long)cols, shape_str(x).c_str(),
                        (unsigned long long)rows, (unsigned long long)cols, shape_str(w).c_str());
        }
    }
    if (!(epsilon > 0.0f)) return fail(MG_SHAPE_UNSUPPORTED, "RMSNorm epsilon must be positive");
    Buffer* o;
    MG_TRY(output_for(d, MG_F32, x->rank, x->shape, out, &o));
    r->x = (const float*)x->ptr;
    r->w = w ? (const float*)w->ptr : nullptr;
    r->out = (float*)o->ptr;
    r->rows = rows;
    r->cols = cols;
    r->w_stride = w_stride;
    r->eps = epsilon;
    return MG_OK;
}
}  // namespace mg

extern "C" {

mg_status mg_rmsnorm(mg_device* h, const mg_buffer* xh, const mg_buffer* wh, float epsilon, uint64_t head_count,
                     uint64_t head_dimension, mg_buffer** out) {
    k::RmsArgs r;
    MG_TRY(rmsnorm_plan(h, xh, wh, epsilon, head_count, head_dimension, out, &r));
    return k::rmsnorm(dev(h), r.x, r.w, r.out, r.rows, r.cols, r.w_stride, r.eps);
}

}  // extern "C"

namespace mg {
// src/kernels.rs:2278-2325
mg_status kv_write_plan(mg_device* h, mg_buffer* sh, const mg_buffer* rh, uint64_t row_offset, k::KvWriteArgs* a) {
    MG_TRY(device_check(h));
    MG_TRY(need(sh, "store"));
    MG_TRY(need(rh, "rows"));
    Device* d = dev(h);
    Buffer* store = buf(sh);
    const Buffer* rows = buf(rh);
    MG_TRY(same_device(d, store));
    MG_TRY(same_device(d, rows));
    MG_TRY(require_f32(store, "kv-write"));
    MG_TRY(require_f32(rows, "kv-write"));
    uint64_t capacity, width, count, row_width;
    MG_TRY(rows_cols(store, &capacity, &width));
    MG_TRY(rows_cols(rows, &count, &row_width));
    if (row_width != width)
        return fail(MG_SHAPE_UNSUPPORTED, "kv-write rows have width %llu, the store %llu", (unsigned long long)row_width,
                    (unsigned long long)width);
    if (row_offset > capacity || count > capacity - row_offset)
        return fail(MG_SHAPE_UNSUPPORTED, "kv-write of %llu rows at %llu exceeds the store's %llu rows",
                    (unsigned long long)count, (unsigned long long)row_offset, (unsigned long long)capacity);
    a->rows = (const float*)rows->ptr;
    a->store = (float*)store->ptr;
    a->count = count;
    a->width = width;
    a->row_offset = row_offset;
    a->capacity = capacity;
    a->step = nullptr;
    return MG_OK;
}
}  // namespace mg

extern "C" {

mg_status mg_kv_write(mg_device* h, mg_buffer* store, const mg_buffer* rows, uint64_t row_offset) {
    k::KvWriteArgs a;
    MG_TRY(kv_write_plan(h, store, rows, row_offset, &a));
    buffer_drop_prep(buf(store));  // its contents change
    return k::kv_write(dev(h), a);
}

// src/kernels.rs:4224-4355
mg_status mg_rope(mg_device* h, const mg_buffer* xh, const mg_rope_params* pp, mg_buffer** out) {
    k::RopeArgs a;
    MG_TRY(mg::rope_plan(h, xh, pp, out, &a));
    return k::rope(dev(h), (const float*)buf(xh)->ptr, (float*)buf(*out)->ptr, a);
}

}  // extern "C"

namespace mg {
// src/kernels.rs:4224-4355: everything a rope does but the launch.
mg_status rope_plan(mg_device* h, const mg_buffer* xh, const mg_rope_params* pp, mg_buffer** out, k::RopeArgs* ap) {
    MG_TRY(device_check(h));
    MG_TRY(need(xh, "input"));
    if (!pp) return fail(MG_INVALID_ARGUMENT, "null rope parameters");
    Device* d = dev(h);
    const Buffer* x = buf(xh);
    MG_TRY(same_device(d, x));
    MG_TRY(require_f32(x, "rope"));
    const mg_rope_params& p = *pp;
    if (p.banded_factor > 0.0f && p.yarn_factor > 0.0f)
        return fail(MG_SHAPE_UNSUPPORTED, "RoPE takes one frequency scaling, not banded and YaRN together");
    uint64_t rows, cols;
    MG_TRY(rows_cols(x, &rows, &cols));
    if (p.head_count == 0 || cols % p.head_count != 0)
        return fail(MG_SHAPE_UNSUPPORTED, "RoPE head_count %llu must be positive and evenly divide the row width %llu",
                    (unsigned long long)p.head_count, (unsigned long long)cols);
    const uint64_t head_width = cols / p.head_count;
    if (p.dimension == 0 || p.dimension % 2 != 0 || p.dimension > head_width)
        return fail(MG_SHAPE_UNSUPPORTED,
                    "RoPE dimension %llu must be positive, even, and at most the head width %llu",
                    (unsigned long long)p.dimension, (unsigned long long)head_width);
    if (!std::isfinite(p.base) || p.base <= 0.0f) return fail(MG_SHAPE_UNSUPPORTED, "RoPE base must be finite and positive");
    if (!std::isfinite(p.scale) || p.scale <= 0.0f)
        return fail(MG_SHAPE_UNSUPPORTED, "RoPE scale must be finite and positive");
    if (p.pairing != 0 && p.pairing != 1) return fail(MG_SHAPE_UNSUPPORTED, "RoPE pairing %d is not implemented", p.pairing);
    const uint64_t half = p.dimension / 2;
    // src/kernels.rs:7184-7202: rows * head_count * half must not overflow.
    if (p.head_count != 0 && half != 0 &&
        (rows > UINT64_MAX / p.head_count || rows * p.head_count > UINT64_MAX / half))
        return fail(MG_SHAPE_UNSUPPORTED, "RoPE launch size overflows: rows %llu * head_count %llu * half %llu",
                    (unsigned long long)rows, (unsigned long long)p.head_count, (unsigned long long)half);
    if (half * sizeof(float2) > 200 * 1024)
        return fail(MG_SHAPE_UNSUPPORTED, "RoPE dimension %llu exceeds the supported 51200 pairs", (unsigned long long)p.dimension);
    Buffer* o;
    MG_TRY(output_for(d, MG_F32, x->rank, x->shape, out, &o));
    k::RopeArgs a;
    a.rows = rows;
    a.cols = cols;
    a.half = half;
    a.dimension = p.dimension;
    a.position_offset = p.position_offset;
    a.head_count = p.head_count;
    a.rotated_pairs = p.rotated_pairs < half ? p.rotated_pairs : half;
    a.base = p.base;
    a.scale = p.scale;
    a.banded_factor = p.banded_factor;
    a.low_freq_factor = p.low_freq_factor;
    a.high_freq_factor = p.high_freq_factor;
    a.original_context_length = p.original_context_length;
    a.yarn_factor = p.yarn_factor;
    a.yarn_low = p.yarn_low;
    a.yarn_high = p.yarn_high;
    a.amplitude = p.yarn_factor > 0.0f ? p.amplitude : 1.0f;
    a.half_split = p.pairing;
    *ap = a;
    return MG_OK;
}
}  // namespace mg

extern "C" {

// src/kernels.rs:4357-4386
// src/kernels.rs:1964-1967: a packed weight's logical matrix as f32.
mg_status mg_dequantize_q8(mg_device* h, const mg_buffer* ph, mg_buffer** out) {
    MG_TRY(device_check(h));
    MG_TRY(need(ph, "packed weight"));
    Device* d = dev(h);
    const Buffer* p = buf(ph);
    MG_TRY(same_device(d, p));
    if (p->dtype != MG_Q8_0) return fail(MG_DTYPE_UNSUPPORTED, "not a packed weight");
    Buffer* o;
    MG_TRY(output_for(d, MG_F32, 2, p->shape, out, &o));
    return k::q8_dequantize(d, p, (float*)o->ptr, false);
}

// src/kernels.rs:4441-4488: the column of one logits row with the highest score over the
// temperature, among finite scores outside the excluded ranges; *found = 0 when none is eligible.
mg_status mg_greedy_select(mg_device* h, const mg_buffer* lh, uint64_t row, const uint64_t* excluded,
                           uint32_t excluded_count, float temperature, int* found, uint64_t* column) {
    MG_TRY(device_check(h));
    MG_TRY(need(lh, "logits"));
    if (!found || !column || (excluded_count && !excluded)) return fail(MG_INVALID_ARGUMENT, "null argument");
    *found = 0;
    *column = 0;
    Device* d = dev(h);
    const Buffer* l = buf(lh);
    MG_TRY(same_device(d, l));
    MG_TRY(require_f32(l, "greedy selection's logits"));
    if (l->rank < 1) return fail(MG_SHAPE_UNSUPPORTED, "logits have no columns");
    const uint64_t cols = l->shape[l->rank - 1];
    const uint64_t rows = l->count / (cols ? cols : 1);
    if (cols == 0 || row >= rows || cols > 0xFFFFFFFFull)
        return fail(MG_SHAPE_UNSUPPORTED, "no logits row %llu of %llu rows of %llu columns", (unsigned long long)row,
                    (unsigned long long)rows, (unsigned long long)cols);
    if (d->capturing) return fail(MG_CAPTURE_UNSUPPORTED, "greedy selection reads its result on the host and cannot be captured");
    uint64_t key = 0;
    MG_TRY(k::greedy_select(d, (const float*)l->ptr + row * cols, cols, excluded, excluded_count, temperature, &key));
    if (key) {
        *found = 1;
        *column = 0xFFFFFFFFull - (key & 0xFFFFFFFFull);
    }
    return MG_OK;
}

mg_status mg_softmax(mg_device* h, const mg_buffer* xh, mg_buffer** out) {
    MG_TRY(device_check(h));
    MG_TRY(need(xh, "input"));
    Device* d = dev(h);
    const Buffer* x = buf(xh);
    MG_TRY(same_device(d, x));
    MG_TRY(require_f32(x, "softmax"));
    uint64_t rows, cols;
    MG_TRY(rows_cols(x, &rows, &cols));
    if (d->capturing) return fail(MG_CAPTURE_UNSUPPORTED, "softmax reads its row flag on the host and cannot be captured");
    Buffer* o;
    MG_TRY(output_for(d, MG_F32, 2, x->shape, out, &o));
    MG_CUDA(cudaMemsetAsync(d->flags + 1, 0, sizeof(int), d->stream), "resetting the softmax flag");
    MG_TRY(k::softmax(d, (const float*)x->ptr, (float*)o->ptr, rows, cols, d->flags + 1));
    int flags[4];
    MG_TRY(read_flags(d, flags));
    if (flags[1]) return fail(MG_EXECUTION_FAILED, "softmax has a row with no finite entry to normalize");
    return MG_OK;
}

mg_status mg_matmul(mg_device* h, const mg_buffer* a, const mg_buffer* b, int ta, int tb, mg_buffer** out) {
    return matmul_impl(h, a, b, nullptr, nullptr, kNone, ta, tb, out);
}

mg_status mg_matmul_bias(mg_device* h, const mg_buffer* a, const mg_buffer* b, const mg_buffer* bias, int ta, int tb,
                         mg_buffer** out) {
    if (!bias) return fail(MG_INVALID_ARGUMENT, "null bias buffer");
    return matmul_impl(h, a, b, nullptr, bias, kRow, ta, tb, out);
}

mg_status mg_matmul_residual(mg_device* h, const mg_buffer* a, const mg_buffer* b, const mg_buffer* residual, int ta,
                             int tb, mg_buffer** out) {
    if (!residual) return fail(MG_INVALID_ARGUMENT, "null residual buffer");
    return matmul_impl(h, a, b, nullptr, residual, kFull, ta, tb, out);
}

mg_status mg_gated_matmul(mg_device* h, const mg_buffer* a, const mg_buffer* gate, const mg_buffer* up, int ta, int tb,
                          mg_buffer** out) {
    if (!up) return fail(MG_INVALID_ARGUMENT, "null up buffer");
    return matmul_impl(h, a, gate, up, nullptr, kNone, ta, tb, out);
}

// src/kernels.rs:6505-6629
}  // extern "C"

namespace mg {
mg_status attention_plan(mg_device* h, const mg_buffer* qh, const mg_buffer* kh, const mg_buffer* vh,
                         const mg_attention_params* pp, mg_buffer** out, k::AttentionArgs* ap) {
    MG_TRY(device_check(h));
    MG_TRY(need(qh, "q"));
    MG_TRY(need(kh, "k"));
    MG_TRY(need(vh, "v"));
    if (!pp) return fail(MG_INVALID_ARGUMENT, "null attention parameters");
    Device* d = dev(h);
    const Buffer* q = buf(qh);
    const Buffer* kb = buf(kh);
    const Buffer* v = buf(vh);
    MG_TRY(same_device(d, q));
    MG_TRY(same_device(d, kb));
    MG_TRY(same_device(d, v));
    MG_TRY(require_f32(q, "attention"));
    MG_TRY(require_f32(kb, "attention"));
    MG_TRY(require_f32(v, "attention"));
    const mg_attention_params& p = *pp;
    const uint64_t head_count = p.head_count, head_dim = p.head_dimension;
    const uint64_t value_dim = p.value_dimension ? p.value_dimension : head_dim;
    if (value_dim == head_dim && !same_shape(kb, v))
        return fail(MG_SHAPE_UNSUPPORTED, "shape mismatch: %s vs %s", shape_str(kb).c_str(), shape_str(v).c_str());
    float scale;
    if (p.has_scale) {
        if (!std::isfinite(p.scale) || !(p.scale > 0.0f))
            return fail(MG_SHAPE_UNSUPPORTED, "attention scale %g must be finite and positive", (double)p.scale);
        scale = p.scale;
    } else {
        scale = 1.0f / sqrtf((float)head_dim);
    }
    const uint64_t kv_heads = p.kv_head_count ? p.kv_head_count : head_count;
    if (head_count == 0 || head_dim == 0 || kv_heads == 0 || value_dim == 0)
        return fail(MG_SHAPE_UNSUPPORTED, "head_count, kv_head_count, and head_dimension must all be positive");
    if (head_count % kv_heads != 0)
        return fail(MG_SHAPE_UNSUPPORTED, "head_count %llu must be an exact multiple of kv_head_count %llu",
                    (unsigned long long)head_count, (unsigned long long)kv_heads);
    if (p.window_size == 0) return fail(MG_SHAPE_UNSUPPORTED, "window_size must be positive; a zero window admits no keys");
    if (p.window_size > 0 && !p.causal)
        return fail(MG_SHAPE_UNSUPPORTED, "window_size is only defined for causal attention");
    uint64_t seq_len, q_model_dim, kv_rows, kv_model_dim, v_rows, v_model_dim;
    MG_TRY(rows_cols(q, &seq_len, &q_model_dim));
    MG_TRY(rows_cols(kb, &kv_rows, &kv_model_dim));
    const uint64_t kv_seq_len = p.key_count >= 0 ? (uint64_t)p.key_count : kv_rows;
    if (kv_seq_len > kv_rows)
        return fail(MG_SHAPE_UNSUPPORTED, "key_count %llu exceeds the %llu rows of K/V", (unsigned long long)kv_seq_len,
                    (unsigned long long)kv_rows);
    if (seq_len > kv_seq_len)
        return fail(MG_SHAPE_UNSUPPORTED, "q sequence length %llu cannot exceed k/v sequence length %llu",
                    (unsigned long long)seq_len, (unsigned long long)kv_seq_len);
    if (head_count * head_dim != q_model_dim)
        return fail(MG_SHAPE_UNSUPPORTED, "head_count * head_dimension must equal q row width %llu, got %llu * %llu",
                    (unsigned long long)q_model_dim, (unsigned long long)head_count, (unsigned long long)head_dim);
    if (kv_heads * head_dim != kv_model_dim)
        return fail(MG_SHAPE_UNSUPPORTED,
                    "kv_head_count * head_dimension must equal k/v row width %llu, got %llu * %llu",
                    (unsigned long long)kv_model_dim, (unsigned long long)kv_heads, (unsigned long long)head_dim);
    MG_TRY(rows_cols(v, &v_rows, &v_model_dim));
    if (v_rows != kv_rows || kv_heads * value_dim != v_model_dim)
        return fail(MG_SHAPE_UNSUPPORTED,
                    "v must hold %llu rows of kv_head_count * value_dimension = %llu * %llu, got %s",
                    (unsigned long long)kv_rows, (unsigned long long)kv_heads, (unsigned long long)value_dim,
                    shape_str(v).c_str());
    const uint64_t shape[2] = {seq_len, head_count * value_dim};
    Buffer* o;
    MG_TRY(output_for(d, MG_F32, 2, shape, out, &o));
    k::AttentionArgs a;
    a.q = (const float*)q->ptr;
    a.k = (const float*)kb->ptr;
    a.v = (const float*)v->ptr;
    a.out = (float*)o->ptr;
    a.seq_len = seq_len;
    a.kv_seq_len = kv_seq_len;
    a.head_count = head_count;
    a.kv_head_count = kv_heads;
    a.head_dim = head_dim;
    a.value_dim = value_dim;
    a.q_model_dim = q_model_dim;
    a.kv_model_dim = kv_model_dim;
    a.v_model_dim = v_model_dim;
    a.causal = p.causal ? 1 : 0;
    a.window = p.window_size > 0 ? p.window_size : -1;
    a.query_position_offset = kv_seq_len - seq_len;
    a.scale = scale;
    a.step = nullptr;
    a.kv_rows = kv_rows;
    *ap = a;
    return MG_OK;
}
}  // namespace mg

extern "C" {

mg_status mg_attention(mg_device* h, const mg_buffer* qh, const mg_buffer* kh, const mg_buffer* vh,
                       const mg_attention_params* pp, mg_buffer** out) {
    k::AttentionArgs a;
    MG_TRY(attention_plan(h, qh, kh, vh, pp, out, &a));
    return k::attention(dev(h), a);
}

}  // extern "C"
