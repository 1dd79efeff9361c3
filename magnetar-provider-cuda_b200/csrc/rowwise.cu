// Row-structured memory-bound kernels: rmsnorm, rope, softmax and the embedding gather.
//
// Each reads its input from HBM once and writes its output once.  The reference runs
// rmsnorm as one 256-thread CTA per row with a shared-memory tree (src/kernels.cu:1103-1138),
// rope as one thread per pair recomputing powf/sinf/cosf for every head
// (src/kernels.cu:1147-1229), softmax as one thread per row over three passes
// (src/kernels.cu:1232-1260) and the embedding as one thread per row copying serially
// (src/kernels.cu:127-176).  Here rows are cached in registers between the reduction and
// the write, reductions are warp shuffles, accesses are 16-byte vectors, and rope computes
// each (row, pair) rotation once for all heads.  The per-element f32 expressions are the
// reference's; only the order of the row reductions differs (a tree instead of a serial sum).
#include "internal.h"
#include "rope.cuh"

namespace mg {
namespace {

__device__ __forceinline__ bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Sum over a CTA of NW warps; every thread gets the total.  `red` holds NW floats.
template <int NW>
__device__ __forceinline__ float block_sum(float v, float* red) {
    v = warp_sum(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = lane < NW ? red[lane] : 0.0f;
    return warp_sum(t);
}
template <int NW>
__device__ __forceinline__ float block_max(float v, float* red) {
    v = warp_max(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = lane < NW ? red[lane] : __int_as_float(0xff800000);
    return warp_max(t);
}

// =====================================================================================
// rmsnorm: y = x * (1 / sqrtf(mean(x^2) + eps)) [* w]   (src/kernels.cu:1118-1137)
// TPR threads per row (32: a warp per row, 256: a CTA per row); each thread caches up to
// VPT float4 of its row so the row is read once.
// =====================================================================================
template <int TPR, int VPT>
__global__ void __launch_bounds__(256) rmsnorm_vec_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                          float* __restrict__ out, uint64_t rows, uint64_t cols,
                                                          uint64_t w_stride, float eps) {
    pdl_enter();
    __shared__ float red[8];
    const int rows_per_cta = 256 / TPR;
    const int sub = threadIdx.x / TPR, t = threadIdx.x % TPR;
    const uint64_t c4 = cols >> 2;
    for (uint64_t row0 = (uint64_t)blockIdx.x * rows_per_cta; row0 < rows; row0 += (uint64_t)gridDim.x * rows_per_cta) {
        const uint64_t row = row0 + sub;
        const bool live = row < rows;
        const float4* in = reinterpret_cast<const float4*>(x + (live ? row : 0) * cols);
        float4 cache[VPT];
        float sum = 0.0f;
#pragma unroll
        for (int j = 0; j < VPT; j++) {
            uint64_t idx = (uint64_t)t + (uint64_t)j * TPR;
            if (live && idx < c4) {
                float4 v = in[idx];
                cache[j] = v;
                sum += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
            }
        }
        for (uint64_t idx = (uint64_t)t + (uint64_t)VPT * TPR; live && idx < c4; idx += TPR) {
            float4 v = in[idx];
            sum += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
        float total;
        if (TPR == 32) total = warp_sum(sum);
        else total = block_sum<TPR / 32>(sum, red);
        if (!live) continue;
        const float scale = 1.0f / sqrtf(total / (float)cols + eps);
        float4* o = reinterpret_cast<float4*>(out + row * cols);
        const float4* wr = w ? reinterpret_cast<const float4*>(w + row * w_stride) : nullptr;
#pragma unroll
        for (int j = 0; j < VPT; j++) {
            uint64_t idx = (uint64_t)t + (uint64_t)j * TPR;
            if (idx < c4) {
                float4 v = cache[j], r;
                if (wr) {
                    float4 g = wr[idx];
                    r = make_float4(v.x * scale * g.x, v.y * scale * g.y, v.z * scale * g.z, v.w * scale * g.w);
                } else {
                    r = make_float4(v.x * scale, v.y * scale, v.z * scale, v.w * scale);
                }
                o[idx] = r;
            }
        }
        for (uint64_t idx = (uint64_t)t + (uint64_t)VPT * TPR; idx < c4; idx += TPR) {
            float4 v = in[idx], r;
            if (wr) {
                float4 g = wr[idx];
                r = make_float4(v.x * scale * g.x, v.y * scale * g.y, v.z * scale * g.z, v.w * scale * g.w);
            } else {
                r = make_float4(v.x * scale, v.y * scale, v.z * scale, v.w * scale);
            }
            o[idx] = r;
        }
    }
}

// Any shape or alignment: one CTA per row, scalar accesses, two reads of the row.
__global__ void __launch_bounds__(256) rmsnorm_scalar_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                             float* __restrict__ out, uint64_t rows, uint64_t cols,
                                                             uint64_t w_stride, float eps) {
    pdl_enter();
    __shared__ float red[8];
    for (uint64_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const float* in = x + row * cols;
        float sum = 0.0f;
        for (uint64_t i = threadIdx.x; i < cols; i += 256) sum += in[i] * in[i];
        const float total = block_sum<8>(sum, red);
        const float scale = 1.0f / sqrtf(total / (float)cols + eps);
        const float* wr = w ? w + row * w_stride : nullptr;
        float* o = out + row * cols;
        for (uint64_t i = threadIdx.x; i < cols; i += 256) o[i] = wr ? in[i] * scale * wr[i] : in[i] * scale;
    }
}

// =====================================================================================
// rope (src/kernels.cu:1183-1228).  One CTA per row at a time: the CTA first evaluates
// the rotation (cos, sin) of each of the row's `half` pairs -- the reference's exact
// per-pair expression -- into shared memory, then rotates every head's pairs with it.
// =====================================================================================
__global__ void __launch_bounds__(256) rope_kernel(const float* __restrict__ x, float* __restrict__ out, RopeK p) {
    pdl_enter();
    extern __shared__ float2 cs[];  // [half]
    for (uint64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
        __syncthreads();
        for (uint64_t pair = threadIdx.x; pair < p.half; pair += blockDim.x) cs[pair] = rope_cs(p, row, pair);
        __syncthreads();
        const float* in = x + row * p.cols;
        float* o = out + row * p.cols;
        if (p.vec && !p.half_split) {
            // Interleaved: a float4 at column c holds pairs c/2 and c/2+1 of one head.
            const uint64_t c4 = p.cols >> 2, hw4 = p.head_width >> 2;
            for (uint64_t i = threadIdx.x; i < c4; i += blockDim.x) {
                const uint64_t col = (i % hw4) << 2;
                float4 v = reinterpret_cast<const float4*>(in)[i];
                if (col < p.dimension) {
                    float2 r0 = cs[col >> 1], r1 = cs[(col >> 1) + 1];
                    float4 y;
                    y.x = v.x * r0.x - v.y * r0.y;
                    y.y = v.x * r0.y + v.y * r0.x;
                    y.z = v.z * r1.x - v.w * r1.y;
                    y.w = v.z * r1.y + v.w * r1.x;
                    v = y;
                }
                reinterpret_cast<float4*>(o)[i] = v;
            }
        } else if (p.vec) {
            // Half-split: columns [c, c+4) pair with [c+half, c+half+4).
            const uint64_t hw4 = p.head_width >> 2, h4 = p.half >> 2;
            const uint64_t per_row = p.head_count * hw4;
            for (uint64_t i = threadIdx.x; i < per_row; i += blockDim.x) {
                const uint64_t head = i / hw4, q = i % hw4;
                const uint64_t base = head * p.head_width;
                const uint64_t col = q << 2;
                if (col >= p.dimension) {
                    reinterpret_cast<float4*>(o + base)[q] = reinterpret_cast<const float4*>(in + base)[q];
                } else if (q < h4) {
                    float4 a = reinterpret_cast<const float4*>(in + base)[q];
                    float4 b = reinterpret_cast<const float4*>(in + base + p.half)[q];
                    float2 r0 = cs[col], r1 = cs[col + 1], r2 = cs[col + 2], r3 = cs[col + 3];
                    float4 ya, yb;
                    ya.x = a.x * r0.x - b.x * r0.y; yb.x = a.x * r0.y + b.x * r0.x;
                    ya.y = a.y * r1.x - b.y * r1.y; yb.y = a.y * r1.y + b.y * r1.x;
                    ya.z = a.z * r2.x - b.z * r2.y; yb.z = a.z * r2.y + b.z * r2.x;
                    ya.w = a.w * r3.x - b.w * r3.y; yb.w = a.w * r3.y + b.w * r3.x;
                    reinterpret_cast<float4*>(o + base)[q] = ya;
                    reinterpret_cast<float4*>(o + base + p.half)[q] = yb;
                }
            }
        } else {
            // Any shape: one thread per (head, pair); the pass-through columns are copied.
            const uint64_t per_row = p.head_count * p.half;
            for (uint64_t i = threadIdx.x; i < per_row; i += blockDim.x) {
                const uint64_t head = i / p.half, pair = i % p.half;
                const uint64_t base = head * p.head_width;
                const uint64_t first = p.half_split ? base + pair : base + 2 * pair;
                const uint64_t second = p.half_split ? base + pair + p.half : base + 2 * pair + 1;
                float2 r = cs[pair];
                float a = in[first], b = in[second];
                o[first] = a * r.x - b * r.y;
                o[second] = a * r.y + b * r.x;
            }
            if (p.dimension != p.head_width) {
                const uint64_t rest = p.head_width - p.dimension;
                for (uint64_t i = threadIdx.x; i < p.head_count * rest; i += blockDim.x) {
                    const uint64_t c = (i / rest) * p.head_width + p.dimension + i % rest;
                    o[c] = in[c];
                }
            }
        }
    }
}

// A warp per row for 16-byte-aligned rows: lane j owns float4 column j (and j + 32, ...) of
// every head, evaluates the rotation of that float4's pairs once for the row, and applies it
// to the same float4 of all heads -- each head's 32 float4 form one coalesced 512-byte access.
__global__ void __launch_bounds__(256) rope_warp_kernel(const float* __restrict__ x, float* __restrict__ out, RopeK p) {
    pdl_enter();
    const int lane = threadIdx.x & 31;
    const uint64_t warps = (uint64_t)gridDim.x * 8;
    const uint64_t hw4 = p.head_width >> 2;
    for (uint64_t row = (uint64_t)blockIdx.x * 8 + (threadIdx.x >> 5); row < p.rows; row += warps) {
        const float4* in = reinterpret_cast<const float4*>(x + row * p.cols);
        float4* o = reinterpret_cast<float4*>(out + row * p.cols);
        for (uint64_t q = lane; q < hw4; q += 32) {
            const uint64_t col = q << 2;
            if (!p.half_split) {
                if (col < p.dimension) {
                    const float2 r0 = rope_cs(p, row, col >> 1), r1 = rope_cs(p, row, (col >> 1) + 1);
                    for (uint64_t h = 0; h < p.head_count; h++) {
                        float4 v = in[h * hw4 + q], y;
                        y.x = v.x * r0.x - v.y * r0.y;
                        y.y = v.x * r0.y + v.y * r0.x;
                        y.z = v.z * r1.x - v.w * r1.y;
                        y.w = v.z * r1.y + v.w * r1.x;
                        o[h * hw4 + q] = y;
                    }
                } else {
                    for (uint64_t h = 0; h < p.head_count; h++) o[h * hw4 + q] = in[h * hw4 + q];
                }
            } else {
                if (col >= p.dimension) {
                    for (uint64_t h = 0; h < p.head_count; h++) o[h * hw4 + q] = in[h * hw4 + q];
                } else if (col < p.half) {
                    const uint64_t q2 = q + (p.half >> 2);
                    const float2 r0 = rope_cs(p, row, col), r1 = rope_cs(p, row, col + 1);
                    const float2 r2 = rope_cs(p, row, col + 2), r3 = rope_cs(p, row, col + 3);
                    for (uint64_t h = 0; h < p.head_count; h++) {
                        const float4 a = in[h * hw4 + q], b = in[h * hw4 + q2];
                        float4 ya, yb;
                        ya.x = a.x * r0.x - b.x * r0.y; yb.x = a.x * r0.y + b.x * r0.x;
                        ya.y = a.y * r1.x - b.y * r1.y; yb.y = a.y * r1.y + b.y * r1.x;
                        ya.z = a.z * r2.x - b.z * r2.y; yb.z = a.z * r2.y + b.z * r2.x;
                        ya.w = a.w * r3.x - b.w * r3.y; yb.w = a.w * r3.y + b.w * r3.x;
                        o[h * hw4 + q] = ya;
                        o[h * hw4 + q2] = yb;
                    }
                }
            }
        }
    }
}

// =====================================================================================
// softmax rows (src/kernels.cu:1243-1259): out = expf(x - max) / sum(expf(x - max)).
// A row whose max is not finite raises the device flag and is written as zeros.
// Warp per row with VPL float4 per lane cached (cols <= 128 * VPL); larger rows take a
// CTA per row reading the row three times (L2-resident between passes).
// =====================================================================================
template <int VPL>
__global__ void __launch_bounds__(256) softmax_warp_kernel(const float* __restrict__ x, float* __restrict__ out,
                                                           uint64_t rows, uint64_t cols, int* flag) {
    pdl_enter();
    const int lane = threadIdx.x & 31;
    const uint64_t warps = (uint64_t)gridDim.x * 8;
    const uint64_t c4 = cols >> 2;
    for (uint64_t row = (uint64_t)blockIdx.x * 8 + (threadIdx.x >> 5); row < rows; row += warps) {
        const float4* in = reinterpret_cast<const float4*>(x + row * cols);
        float4 v[VPL];
        float mx = __int_as_float(0xff800000);
#pragma unroll
        for (int j = 0; j < VPL; j++) {
            uint64_t idx = lane + 32 * j;
            if (idx < c4) {
                v[j] = in[idx];
                mx = fmaxf(mx, fmaxf(fmaxf(v[j].x, v[j].y), fmaxf(v[j].z, v[j].w)));
            }
        }
        mx = warp_max(mx);
        float4* o = reinterpret_cast<float4*>(out + row * cols);
        if (!isfinite(mx)) {
            if (lane == 0) atomicExch(flag, 1);
#pragma unroll
            for (int j = 0; j < VPL; j++)
                if (lane + 32 * j < c4) o[lane + 32 * j] = make_float4(0.f, 0.f, 0.f, 0.f);
            continue;
        }
        float sum = 0.0f;
#pragma unroll
        for (int j = 0; j < VPL; j++) {
            if (lane + 32 * j < c4) {
                v[j].x = expf(v[j].x - mx);
                v[j].y = expf(v[j].y - mx);
                v[j].z = expf(v[j].z - mx);
                v[j].w = expf(v[j].w - mx);
                sum += (v[j].x + v[j].y) + (v[j].z + v[j].w);
            }
        }
        sum = warp_sum(sum);
#pragma unroll
        for (int j = 0; j < VPL; j++)
            if (lane + 32 * j < c4)
                o[lane + 32 * j] = make_float4(v[j].x / sum, v[j].y / sum, v[j].z / sum, v[j].w / sum);
    }
}

__global__ void __launch_bounds__(256) softmax_block_kernel(const float* __restrict__ x, float* __restrict__ out,
                                                            uint64_t rows, uint64_t cols, int* flag) {
    pdl_enter();
    __shared__ float red[8];
    for (uint64_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const float* in = x + row * cols;
        float* o = out + row * cols;
        float mx = __int_as_float(0xff800000);
        for (uint64_t i = threadIdx.x; i < cols; i += 256) mx = fmaxf(mx, in[i]);
        mx = block_max<8>(mx, red);
        if (!isfinite(mx)) {
            if (threadIdx.x == 0) atomicExch(flag, 1);
            for (uint64_t i = threadIdx.x; i < cols; i += 256) o[i] = 0.0f;
            continue;
        }
        float sum = 0.0f;
        for (uint64_t i = threadIdx.x; i < cols; i += 256) sum += expf(in[i] - mx);
        sum = block_sum<8>(sum, red);
        for (uint64_t i = threadIdx.x; i < cols; i += 256) o[i] = expf(in[i] - mx) / sum;
    }
}

// =====================================================================================
// embedding (src/kernels.cu:140-175): a warp per id copies the table row with 16-byte
// accesses.  An id that is negative, non-integer or >= vocab raises the flag and leaves
// its row unwritten.  `has_scale` multiplies the copied row (the executor's `scale`).
// =====================================================================================
__global__ void __launch_bounds__(256) embedding_kernel(const float* __restrict__ table, const float* __restrict__ ids,
                                                        float* __restrict__ out, uint64_t dim, uint64_t num_ids,
                                                        uint64_t vocab, int* flag, int has_scale, float scale,
                                                        int vec) {
    pdl_enter();
    const int lane = threadIdx.x & 31;
    const uint64_t warps = (uint64_t)gridDim.x * 8;
    for (uint64_t row = (uint64_t)blockIdx.x * 8 + (threadIdx.x >> 5); row < num_ids; row += warps) {
        const float raw = ids[row];
        if (raw < 0.0f || raw != floorf(raw) || !(raw < (float)vocab && (uint64_t)raw < vocab)) {
            if (lane == 0) atomicExch(flag, 1);
            continue;
        }
        const uint64_t id = (uint64_t)raw;
        const float* src = table + id * dim;
        float* dst = out + row * dim;
        if (vec) {
            const float4* s4 = reinterpret_cast<const float4*>(src);
            float4* d4 = reinterpret_cast<float4*>(dst);
            for (uint64_t i = lane; i < (dim >> 2); i += 32) {
                float4 v = s4[i];
                if (has_scale) v = make_float4(v.x * scale, v.y * scale, v.z * scale, v.w * scale);
                d4[i] = v;
            }
        } else {
            for (uint64_t i = lane; i < dim; i += 32) dst[i] = has_scale ? src[i] * scale : src[i];
        }
    }
}

// An embedding then an rmsnorm of its rows, fused (the step capture's fusion of the two nodes):
// a warp per id copies the table row to x and writes rmsnorm(x) to h.  The row is the
// embedding kernel's (scaled the same way) and the normalisation is rmsnorm_vec_kernel<32, 8>'s
// -- the same sums in the same order -- so both outputs equal the two separate launches'.
// dim % 4 == 0, dim <= 1024, 16-byte aligned rows.
__global__ void __launch_bounds__(256) embedding_rmsnorm_kernel(const float* __restrict__ table,
                                                                const float* __restrict__ ids, float* __restrict__ x,
                                                                uint64_t dim, uint64_t num_ids, uint64_t vocab,
                                                                int* flag, int has_scale, float scale,
                                                                const float* __restrict__ w, uint64_t w_stride,
                                                                float* __restrict__ h, float eps) {
    pdl_enter();
    const int lane = threadIdx.x & 31;
    const uint64_t warps = (uint64_t)gridDim.x * 8, c4 = dim >> 2;
    for (uint64_t row = (uint64_t)blockIdx.x * 8 + (threadIdx.x >> 5); row < num_ids; row += warps) {
        const float raw = ids[row];
        if (raw < 0.0f || raw != floorf(raw) || !(raw < (float)vocab && (uint64_t)raw < vocab)) {
            if (lane == 0) atomicExch(flag, 1);
            continue;
        }
        const float4* src = reinterpret_cast<const float4*>(table + (uint64_t)raw * dim);
        float4* xo = reinterpret_cast<float4*>(x + row * dim);
        float4 cache[8];
        float sum = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const uint64_t idx = (uint64_t)lane + (uint64_t)j * 32;
            if (idx < c4) {
                float4 v = src[idx];
                if (has_scale) v = make_float4(v.x * scale, v.y * scale, v.z * scale, v.w * scale);
                xo[idx] = v;
                cache[j] = v;
                sum += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
            }
        }
        const float total = warp_sum(sum);
        const float inv = 1.0f / sqrtf(total / (float)dim + eps);
        float4* ho = reinterpret_cast<float4*>(h + row * dim);
        const float4* wr = w ? reinterpret_cast<const float4*>(w + row * w_stride) : nullptr;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const uint64_t idx = (uint64_t)lane + (uint64_t)j * 32;
            if (idx < c4) {
                const float4 v = cache[j];
                float4 r;
                if (wr) {
                    const float4 g = wr[idx];
                    r = make_float4(v.x * inv * g.x, v.y * inv * g.y, v.z * inv * g.z, v.w * inv * g.w);
                } else {
                    r = make_float4(v.x * inv, v.y * inv, v.z * inv, v.w * inv);
                }
                ho[idx] = r;
            }
        }
    }
}

inline unsigned cap_grid(const Device* d, uint64_t want, unsigned per_sm) {
    uint64_t cap = (uint64_t)d->sm_count * per_sm;
    if (want > cap) want = cap;
    return (unsigned)(want ? want : 1);
}

inline bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }


// ---- greedy selection (src/kernels.cu:1808-1866, src/kernels.rs:4441-4488) ----------------------
// Each eligible column of the logits row (raw score finite, outside every excluded [start, end)
// range) is one 64-bit key: the score after the temperature division (as is when the temperature
// is 0; -0 taken as +0) mapped so unsigned order is float order, above the complement of the
// column -- the largest key is the highest score, ties going to the lowest column, whatever order
// threads and CTAs run in.  CTAs fold their largest key into words[0] with atomicMax; the last CTA
// to finish (a ticket in words[1]) moves the result to words[2] and leaves words[0..1] zero for
// the next call, so one launch does the whole reduction.
constexpr int kInlineRanges = 16;
struct GreedyArgs {
    const float* row;
    uint64_t cols;
    const uint64_t* ranges;  // [2 * count] when count > kInlineRanges
    uint64_t inline_ranges[2 * kInlineRanges];
    uint32_t count;
    float temperature;
    unsigned long long* words;  // [0] running max, [1] ticket (low 32 bits), [2] result
};

__device__ __forceinline__ unsigned long long greedy_key(const GreedyArgs& p, uint64_t i, float raw) {
    if (!isfinite(raw)) return 0ull;
    for (uint32_t r = 0; r < p.count; r++) {
        const uint64_t lo = p.count <= kInlineRanges ? p.inline_ranges[2 * r] : p.ranges[2 * r];
        const uint64_t hi = p.count <= kInlineRanges ? p.inline_ranges[2 * r + 1] : p.ranges[2 * r + 1];
        if (i >= lo && i < hi) return 0ull;
    }
    float v = p.temperature != 0.0f ? raw / p.temperature : raw;
    if (v == 0.0f) v = 0.0f;
    const uint32_t bits = __float_as_uint(v);
    const uint32_t ordered = (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
    return ((unsigned long long)ordered << 32) | (0xFFFFFFFFull - (i & 0xFFFFFFFFull));
}

__global__ void __launch_bounds__(256) greedy_select_kernel(const __grid_constant__ GreedyArgs p) {
    pdl_enter();
    unsigned long long key = 0ull;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (; i + 3 * stride < p.cols; i += 4 * stride) {  // four loads in flight
        float v[4];
#pragma unroll
        for (int u = 0; u < 4; u++) v[u] = __ldg(p.row + i + u * stride);
#pragma unroll
        for (int u = 0; u < 4; u++) key = max(key, greedy_key(p, i + u * stride, v[u]));
    }
    for (; i < p.cols; i += stride) key = max(key, greedy_key(p, i, __ldg(p.row + i)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) key = max(key, __shfl_xor_sync(0xFFFFFFFFu, key, o));
    __shared__ unsigned long long warp_keys[8];
    __shared__ bool last;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) warp_keys[warp] = key;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); w++) key = max(key, warp_keys[w]);
        if (key) atomicMax(&p.words[0], key);
        __threadfence();
        last = atomicAdd(&p.words[1], 1ull) == gridDim.x - 1;
        if (last) {
            p.words[2] = atomicExch(&p.words[0], 0ull);
            p.words[1] = 0ull;
        }
    }
}

}  // namespace

namespace k {

mg_status rmsnorm(Device* d, const float* x, const float* w, float* out, uint64_t rows, uint64_t cols,
                  uint64_t w_stride, float eps) {
    const bool vec = cols % 4 == 0 && a16(x) && a16(out) && (!w || (a16(w) && w_stride % 4 == 0));
    if (!vec) {
        enqueue(d, rmsnorm_scalar_kernel, cap_grid(d, rows, 8), 256, 0, x, w, out, rows, cols, w_stride, eps);
    } else if (cols <= 1024) {
        // a warp per row, up to 8 float4 per lane
        enqueue(d, rmsnorm_vec_kernel<32, 8>, cap_grid(d, (rows + 7) / 8, 8), 256, 0, x, w, out, rows, cols,
                                                                                          w_stride, eps);
    } else {
        // a CTA per row, up to 8 float4 per thread (rows of up to 8192 read once)
        enqueue(d, rmsnorm_vec_kernel<256, 8>, cap_grid(d, rows, 8), 256, 0, x, w, out, rows, cols, w_stride, eps);
    }
    return launched(d, "rmsnorm kernel launch");
}

mg_status rope(Device* d, const float* x, float* out, const RopeArgs& a) {
    RopeK p;
    p.rows = a.rows;
    p.cols = a.cols;
    p.half = a.half;
    p.dimension = a.dimension;
    p.position_offset = a.position_offset;
    p.step = a.step;
    p.head_count = a.head_count;
    p.head_width = a.cols / a.head_count;
    p.rotated_pairs = a.rotated_pairs;
    p.base = a.base;
    p.scale = a.scale;
    p.banded_factor = a.banded_factor;
    p.low_freq_factor = a.low_freq_factor;
    p.high_freq_factor = a.high_freq_factor;
    p.original_context_length = a.original_context_length;
    p.yarn_factor = a.yarn_factor;
    p.yarn_low = a.yarn_low;
    p.yarn_high = a.yarn_high;
    p.amplitude = a.amplitude;
    p.half_split = a.half_split;
    bool vec = a16(x) && a16(out) && p.head_width % 4 == 0;
    if (p.half_split) vec = vec && p.half % 4 == 0;
    else vec = vec && p.dimension % 4 == 0;
    p.vec = vec ? 1 : 0;
    if (p.vec) {
        enqueue(d, rope_warp_kernel, cap_grid(d, (a.rows + 7) / 8, 8), 256, 0, x, out, p);
        return launched(d, "rope kernel launch");
    }
    size_t smem = p.half * sizeof(float2);
    if (smem > 48 * 1024) {
        MG_CUDA(cudaFuncSetAttribute(rope_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                "configuring rope shared memory");
    }
    enqueue(d, rope_kernel, cap_grid(d, a.rows, 8), 256, smem, x, out, p);
    return launched(d, "rope kernel launch");
}

mg_status softmax(Device* d, const float* x, float* out, uint64_t rows, uint64_t cols, int* flag) {
    const bool vec = cols % 4 == 0 && a16(x) && a16(out);
    const unsigned grid = cap_grid(d, (rows + 7) / 8, 8);
    if (vec && cols <= 128) enqueue(d, softmax_warp_kernel<1>, grid, 256, 0, x, out, rows, cols, flag);
    else if (vec && cols <= 256) enqueue(d, softmax_warp_kernel<2>, grid, 256, 0, x, out, rows, cols, flag);
    else if (vec && cols <= 512) enqueue(d, softmax_warp_kernel<4>, grid, 256, 0, x, out, rows, cols, flag);
    else if (vec && cols <= 1024) enqueue(d, softmax_warp_kernel<8>, grid, 256, 0, x, out, rows, cols, flag);
    else if (vec && cols <= 2048) enqueue(d, softmax_warp_kernel<16>, grid, 256, 0, x, out, rows, cols, flag);
    else enqueue(d, softmax_block_kernel, cap_grid(d, rows, 8), 256, 0, x, out, rows, cols, flag);
    return launched(d, "softmax kernel launch");
}

mg_status embedding(Device* d, const float* table, const float* ids, float* out, uint64_t dim, uint64_t num_ids,
                    uint64_t vocab, int* flag, int has_scale, float scale) {
    int vec = dim % 4 == 0 && a16(table) && a16(out);
    enqueue(d, embedding_kernel, cap_grid(d, (num_ids + 7) / 8, 8), 256, 0, table, ids, out, dim, num_ids, vocab,
                                                                                flag, has_scale, scale, vec);
    return launched(d, "embedding kernel launch");
}

mg_status embedding_run(Device* d, const EmbedArgs& e, int* flag) {
    if (e.packed) return q8_embedding(d, e.packed, e.ids, e.out, e.num_ids, flag, e.has_scale, e.scale);
    return embedding(d, e.table, e.ids, e.out, e.dim, e.num_ids, e.vocab, flag, e.has_scale, e.scale);
}

bool embedding_rmsnorm_eligible(const EmbedArgs& e, const RmsArgs& r) {
    return !e.packed && r.x == e.out && r.out != e.out && r.rows == e.num_ids && r.cols == e.dim && e.dim % 4 == 0 &&
           e.dim <= 1024 && a16(e.table) && a16(e.out) && a16(r.out) &&
           (!r.w || (a16(r.w) && (r.w_stride == 0 || r.w_stride == e.dim)));
}

mg_status embedding_rmsnorm(Device* d, const EmbedArgs& e, const RmsArgs& r, int* flag) {
    enqueue(d, embedding_rmsnorm_kernel, cap_grid(d, (e.num_ids + 7) / 8, 8), 256, 0, e.table, e.ids, e.out, e.dim,
            e.num_ids, e.vocab, flag, e.has_scale, e.scale, r.w, r.w_stride, r.out, r.eps);
    return launched(d, "embedding + rmsnorm kernel launch");
}

mg_status greedy_select(Device* d, const float* row, uint64_t cols, const uint64_t* excluded, uint32_t count,
                        float temperature, uint64_t* key) {
    GreedyArgs p{};
    p.row = row;
    p.cols = cols;
    p.count = count;
    p.temperature = temperature;
    p.words = reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(d->flags) + 64);
    void* staged = nullptr;
    if (count <= (uint32_t)kInlineRanges) {
        for (uint32_t r = 0; r < 2 * count; r++) p.inline_ranges[r] = excluded[r];
    } else {
        MG_TRY(device_alloc(d, 2 * (size_t)count * sizeof(uint64_t), &staged));
        cudaError_t e = cudaMemcpyAsync(staged, excluded, 2 * (size_t)count * sizeof(uint64_t), cudaMemcpyHostToDevice, d->stream);
        if (e != cudaSuccess) {
            device_free(d, staged);
            return from_cuda(e, "uploading the excluded ranges");
        }
        p.ranges = static_cast<const uint64_t*>(staged);
    }
    uint64_t blocks = (cols + 1023) / 1024;
    if (blocks > (uint64_t)d->sm_count) blocks = (uint64_t)d->sm_count;
    enqueue(d, greedy_select_kernel, (unsigned)(blocks ? blocks : 1), 256, 0, p);
    mg_status s = launched(d, "greedy selection launch");
    if (staged) device_free(d, staged);
    MG_TRY(s);
    uint64_t* host = reinterpret_cast<uint64_t*>(d->host_flags) + 4;  // bytes 32..39 of the pinned words
    MG_CUDA(cudaMemcpyAsync(host, reinterpret_cast<char*>(d->flags) + 80, sizeof(uint64_t), cudaMemcpyDeviceToHost, d->stream),
            "reading the selected key");
    MG_CUDA(cudaStreamSynchronize(d->stream), "waiting for the device");
    *key = *host;
    d->downloads.fetch_add(1);
    return MG_OK;
}

}  // namespace k
}  // namespace mg
