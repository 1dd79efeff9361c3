// Memory-bound elementwise kernels: add, bias-add, mul, mul-by-scalar, scale, silu,
// silu-mul, and the half-precision add/mul with their conversions.
//
// The reference launches one thread per element with 32-bit accesses
// (src/kernels.cu:30-117, 1091-1096, 2913-2939).  Here every kernel is a grid-stride loop
// over 16-byte vectors (4 f32 or 8 half values per access) with U independent vectors in
// flight per thread, on a grid sized to fill every SM; a scalar loop finishes a ragged tail
// and serves unaligned views.  Each output element is computed with exactly the
// reference's f32 expression, so results are identical to it.
#include <cuda_fp16.h>

#include "internal.h"

namespace mg {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

__host__ __device__ inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Grid for a grid-stride loop over `items` work items: at most 8 resident CTAs per SM.
inline unsigned grid_for(const Device* d, uint64_t items) {
    uint64_t want = (items + kThreads - 1) / kThreads;
    uint64_t cap = (uint64_t)d->sm_count * 8;
    if (want > cap) want = cap;
    return (unsigned)(want ? want : 1);
}

// ---- the per-element expressions (shared by vector and scalar paths) -------------------
struct AddOp {
    __device__ float operator()(float a, float b) const { return a + b; }
};
struct MulOp {
    __device__ float operator()(float a, float b) const { return a * b; }
};
// src/kernels.cu:64-71: silu(g) * u with silu(v) = v * (1 / (1 + expf(-v)))
struct SiluMulOp {
    __device__ float operator()(float g, float u) const { return (g * (1.0f / (1.0f + expf(-g)))) * u; }
};
struct SiluOp {
    __device__ float operator()(float v) const { return v * (1.0f / (1.0f + expf(-v))); }
};
struct ScaleOp {
    float f;
    __device__ float operator()(float v) const { return v * f; }
};
// The tanh form of GELU in the reference's order of operations (src/kernels.cu:80-86):
// 0.5 x (1 + tanh(sqrt(2 / pi) (x + 0.044715 x^3))), sqrt(2 / pi) as the f32 0.7978846.
struct GeluTanhOp {
    __device__ float operator()(float x) const {
        return 0.5f * x * (1.0f + tanhf(0.7978846f * (x + 0.044715f * x * x * x)));
    }
};
// src/kernels.cu:1079-1084: 1 / (1 + exp(-x))
struct SigmoidOp {
    __device__ float operator()(float x) const { return 1.0f / (1.0f + expf(-x)); }
};
// src/kernels.cu:103-109: cap * tanh(x / cap)
struct SoftcapOp {
    float cap;
    __device__ float operator()(float x) const { return cap * tanhf(x / cap); }
};

template <class Op>
__device__ inline float4 apply2(Op op, float4 a, float4 b) {
    return make_float4(op(a.x, b.x), op(a.y, b.y), op(a.z, b.z), op(a.w, b.w));
}
template <class Op>
__device__ inline float4 apply1(Op op, float4 a) {
    return make_float4(op(a.x), op(a.y), op(a.z), op(a.w));
}

// out[i] = op(a[i], b[i]) over n elements; vec != 0 when all pointers are 16-byte aligned.
template <class Op>
__global__ void __launch_bounds__(kThreads) binary_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                                          float* __restrict__ out, uint64_t n, int vec, Op op) {
    pdl_enter();
    const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    uint64_t tail = 0;
    if (vec) {
        const uint64_t n4 = n >> 2;
        const float4* a4 = reinterpret_cast<const float4*>(a);
        const float4* b4 = reinterpret_cast<const float4*>(b);
        float4* o4 = reinterpret_cast<float4*>(out);
        uint64_t i = tid;
        for (; i + (kUnroll - 1) * stride < n4; i += kUnroll * stride) {
            float4 x[kUnroll], y[kUnroll];
#pragma unroll
            for (int u = 0; u < kUnroll; u++) {
                x[u] = a4[i + u * stride];
                y[u] = b4[i + u * stride];
            }
#pragma unroll
            for (int u = 0; u < kUnroll; u++) o4[i + u * stride] = apply2(op, x[u], y[u]);
        }
        for (; i < n4; i += stride) o4[i] = apply2(op, a4[i], b4[i]);
        tail = n4 << 2;
    }
    for (uint64_t i = tail + tid; i < n; i += stride) out[i] = op(a[i], b[i]);
}

template <class Op>
__global__ void __launch_bounds__(kThreads) unary_kernel(const float* __restrict__ a, float* __restrict__ out,
                                                         uint64_t n, int vec, Op op) {
    pdl_enter();
    const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    uint64_t tail = 0;
    if (vec) {
        const uint64_t n4 = n >> 2;
        const float4* a4 = reinterpret_cast<const float4*>(a);
        float4* o4 = reinterpret_cast<float4*>(out);
        uint64_t i = tid;
        for (; i + (kUnroll - 1) * stride < n4; i += kUnroll * stride) {
            float4 x[kUnroll];
#pragma unroll
            for (int u = 0; u < kUnroll; u++) x[u] = a4[i + u * stride];
#pragma unroll
            for (int u = 0; u < kUnroll; u++) o4[i + u * stride] = apply1(op, x[u]);
        }
        for (; i < n4; i += stride) o4[i] = apply1(op, a4[i]);
        tail = n4 << 2;
    }
    for (uint64_t i = tail + tid; i < n; i += stride) out[i] = op(a[i]);
}

// src/kernels.cu:1091-1096: out[i] = a[i] + bias[i % cols].  One CTA row-block per
// (row, column chunk); the bias chunk is reused for every row the CTA visits.
__global__ void __launch_bounds__(kThreads) bias_add_kernel(const float* __restrict__ a,
                                                            const float* __restrict__ bias,
                                                            float* __restrict__ out, uint64_t cols,
                                                            uint64_t rows, int vec) {
    pdl_enter();
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (vec) {
        const uint64_t c4 = cols >> 2, n4 = rows * c4;
        const float4* a4 = reinterpret_cast<const float4*>(a);
        const float4* b4 = reinterpret_cast<const float4*>(bias);
        float4* o4 = reinterpret_cast<float4*>(out);
        for (uint64_t i = tid; i < n4; i += stride) {
            float4 x = a4[i], y = b4[i % c4];
            o4[i] = make_float4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w);
        }
    } else {
        const uint64_t n = rows * cols;
        for (uint64_t i = tid; i < n; i += stride) out[i] = a[i] + bias[i % cols];
    }
}

// src/kernels.cu:112-117: out[i] = a[i] * b[0]
__global__ void __launch_bounds__(kThreads) mul_scalar_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                                              float* __restrict__ out, uint64_t n, int vec) {
    pdl_enter();
    const float s = b[0];
    const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    uint64_t tail = 0;
    if (vec) {
        const uint64_t n4 = n >> 2;
        const float4* a4 = reinterpret_cast<const float4*>(a);
        float4* o4 = reinterpret_cast<float4*>(out);
        for (uint64_t i = tid; i < n4; i += stride) {
            float4 x = a4[i];
            o4[i] = make_float4(x.x * s, x.y * s, x.z * s, x.w * s);
        }
        tail = n4 << 2;
    }
    for (uint64_t i = tail + tid; i < n; i += stride) out[i] = a[i] * s;
}

// ---- half precision ----------------------------------------------------------------------
// Decoding is exact for every pattern, NaN payloads included (the top 10 / 7 mantissa bits
// land in the f32 mantissa's top bits, as src/half_precision.rs:15-44 specifies).
__device__ __forceinline__ float f16_decode(uint32_t h) {
    const uint32_t sign = (h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    uint32_t mag;
    if (e == 0x1Fu) {
        mag = 0x7F800000u | (m << 13);
    } else if (e != 0) {
        mag = ((e + 112u) << 23) | (m << 13);
    } else {
        // zero or subnormal: m * 2^-24 is exact in f32
        mag = __float_as_uint((float)m * 5.9604644775390625e-08f);
    }
    return __uint_as_float(sign | mag);
}

__device__ __forceinline__ float bf16_decode(uint32_t h) { return __uint_as_float(h << 16); }

// f32 -> f16, round to nearest even (the hardware conversion is IEEE RNE with subnormal
// results and overflow to infinity); NaN keeps sign and top payload bits, a zero payload
// becoming 1 (src/half_precision.rs:53-59).
__device__ __forceinline__ uint32_t f16_encode(float v) {
    const uint32_t bits = __float_as_uint(v);
    if ((bits & 0x7F800000u) == 0x7F800000u && (bits & 0x007FFFFFu) != 0) {
        uint32_t payload = (bits & 0x007FFFFFu) >> 13;
        return ((bits >> 16) & 0x8000u) | 0x7C00u | (payload ? payload : 1u);
    }
    return __half_as_ushort(__float2half_rn(v));
}

// f32 -> bf16 (src/half_precision.rs:107-117): NaN keeps sign and top 7 payload bits
// (0 becoming 0x40); everything else rounds to nearest even on the bit pattern.
__device__ __forceinline__ uint32_t bf16_encode(float v) {
    const uint32_t bits = __float_as_uint(v);
    if ((bits & 0x7F800000u) == 0x7F800000u && (bits & 0x007FFFFFu) != 0) {
        uint32_t m7 = (bits >> 16) & 0x7Fu;
        return ((bits >> 16) & 0x8000u) | 0x7F80u | (m7 ? m7 : 0x40u);
    }
    return (bits + 0x7FFFu + ((bits >> 16) & 1u)) >> 16;
}

template <int DT>
__device__ __forceinline__ float hdecode(uint32_t h) {
    return DT == MG_F16 ? f16_decode(h) : bf16_decode(h);
}
template <int DT>
__device__ __forceinline__ uint32_t hencode(float v) {
    return DT == MG_F16 ? f16_encode(v) : bf16_encode(v);
}

template <int DT, int OP>
__device__ __forceinline__ uint32_t half_op(uint32_t a, uint32_t b) {
    float x = hdecode<DT>(a), y = hdecode<DT>(b);
    return hencode<DT>(OP == 0 ? x + y : x * y);
}

// Two halves packed in 32 bits.  For f16 the packed hardware conversions do the work: the
// decode is exact for every non-NaN pattern, a NaN input makes the f32 op return the
// canonical NaN whatever its payload, and the RNE encode matches the reference for every
// non-NaN result -- so only NaN results need the reference's encoding rule applied.
template <int DT, int OP>
__device__ __forceinline__ uint32_t half_op2(uint32_t a, uint32_t b) {
    if constexpr (DT == MG_F16) {
        const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&a));
        const float2 y = __half22float2(*reinterpret_cast<const __half2*>(&b));
        const float r0 = OP == 0 ? x.x + y.x : x.x * y.x;
        const float r1 = OP == 0 ? x.y + y.y : x.y * y.y;
        const __half2 h = __floats2half2_rn(r0, r1);
        uint32_t bits = *reinterpret_cast<const uint32_t*>(&h);
        if (r0 != r0) bits = (bits & 0xFFFF0000u) | f16_encode(r0);
        if (r1 != r1) bits = (bits & 0x0000FFFFu) | (f16_encode(r1) << 16);
        return bits;
    } else {
        return half_op<DT, OP>(a & 0xFFFFu, b & 0xFFFFu) | (half_op<DT, OP>(a >> 16, b >> 16) << 16);
    }
}

// src/kernels.cu:2913-2939 over 8 halves per 16-byte access.
template <int DT, int OP>
__global__ void __launch_bounds__(kThreads) half_binary_kernel(const uint16_t* __restrict__ a,
                                                               const uint16_t* __restrict__ b,
                                                               uint16_t* __restrict__ out, uint64_t n, int vec) {
    pdl_enter();
    const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    uint64_t tail = 0;
    if (vec) {
        const uint64_t n8 = n >> 3;
        const uint4* a8 = reinterpret_cast<const uint4*>(a);
        const uint4* b8 = reinterpret_cast<const uint4*>(b);
        uint4* o8 = reinterpret_cast<uint4*>(out);
        uint64_t i = tid;
        for (; i + (kUnroll - 1) * stride < n8; i += kUnroll * stride) {
            uint4 x[kUnroll], y[kUnroll];
#pragma unroll
            for (int u = 0; u < kUnroll; u++) {
                x[u] = a8[i + u * stride];
                y[u] = b8[i + u * stride];
            }
#pragma unroll
            for (int u = 0; u < kUnroll; u++) {
                const uint32_t* xs = &x[u].x;
                const uint32_t* ys = &y[u].x;
                uint4 r;
                uint32_t* rs = &r.x;
#pragma unroll
                for (int w = 0; w < 4; w++) rs[w] = half_op2<DT, OP>(xs[w], ys[w]);
                o8[i + u * stride] = r;
            }
        }
        for (; i < n8; i += stride) {
            uint4 x = a8[i], y = b8[i], r;
            const uint32_t* xs = &x.x;
            const uint32_t* ys = &y.x;
            uint32_t* rs = &r.x;
#pragma unroll
            for (int w = 0; w < 4; w++)
                rs[w] = half_op<DT, OP>(xs[w] & 0xFFFFu, ys[w] & 0xFFFFu) |
                        (half_op<DT, OP>(xs[w] >> 16, ys[w] >> 16) << 16);
            o8[i] = r;
        }
        tail = n8 << 3;
    }
    for (uint64_t i = tail + tid; i < n; i += stride) out[i] = (uint16_t)half_op<DT, OP>(a[i], b[i]);
}

// The executor's f32-resident add-half/mul-half (src/executor.rs:1970-2013): each f32
// input is encoded to half and decoded back, the op runs in f32, and the half-encoded
// result is decoded to f32 -- the reference's host round trip, on the device.
template <int DT, int OP>
struct HalfRoundTripOp {
    __device__ float operator()(float a, float b) const {
        float x = hdecode<DT>(hencode<DT>(a)), y = hdecode<DT>(hencode<DT>(b));
        return hdecode<DT>(hencode<DT>(OP == 0 ? x + y : x * y));
    }
};

template <int DT>
__global__ void __launch_bounds__(kThreads) encode_kernel(const float* __restrict__ in, uint16_t* __restrict__ out,
                                                          uint64_t n) {
    pdl_enter();
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = (uint16_t)hencode<DT>(in[i]);
}

template <int DT>
__global__ void __launch_bounds__(kThreads) decode_kernel(const uint16_t* __restrict__ in, float* __restrict__ out,
                                                          uint64_t n) {
    pdl_enter();
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = hdecode<DT>(in[i]);
}

// kv-write (src/kernels.rs:2278-2325): store rows row_offset + step .. + count <- rows, where
// `step` is a captured step's advancing offset read at run time (null: none).
__global__ void __launch_bounds__(kThreads) kv_write_kernel(const float* __restrict__ rows, float* __restrict__ store,
                                                            uint64_t n, uint64_t width, uint64_t row_offset,
                                                            const uint64_t* __restrict__ step, int vec) {
    pdl_enter();
    float* dst = store + (row_offset + (step ? *step : 0)) * width;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t t0 = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (vec) {
        const float4* s4 = reinterpret_cast<const float4*>(rows);
        float4* d4 = reinterpret_cast<float4*>(dst);
        for (uint64_t i = t0; i < n / 4; i += stride) d4[i] = s4[i];
        return;
    }
    for (uint64_t i = t0; i < n; i += stride) dst[i] = rows[i];
}

// row-scale (src/kernels.cu:1066-1077): out[r][c] = x[r][c] * scale[r].
__global__ void __launch_bounds__(kThreads) row_scale_kernel(const float* __restrict__ x, const float* __restrict__ scale,
                                                             float* __restrict__ out, uint64_t rows, uint64_t cols,
                                                             int vec) {
    pdl_enter();
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (vec) {  // cols % 4 == 0
        const uint64_t c4 = cols >> 2, n4 = rows * c4;
        const float4* x4 = reinterpret_cast<const float4*>(x);
        float4* o4 = reinterpret_cast<float4*>(out);
        for (uint64_t i = tid; i < n4; i += stride) {
            const float s = scale[i / c4];
            const float4 v = x4[i];
            o4[i] = make_float4(v.x * s, v.y * s, v.z * s, v.w * s);
        }
        return;
    }
    for (uint64_t i = tid; i < rows * cols; i += stride) out[i] = x[i] * scale[i / cols];
}

// concat across heads (src/kernels.cu:5786-5812): output row r holds `heads` heads, head h being
// a's head h (a_width values) then b's head h -- or b's only head when b_heads == 1.  `vec`:
// both widths multiples of 4 and the buffers 16-byte aligned (16-byte copies).
__global__ void __launch_bounds__(kThreads) concat_heads_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                                                float* __restrict__ out, uint64_t rows, uint64_t heads,
                                                                uint64_t a_width, uint64_t b_width, uint64_t b_heads,
                                                                int vec) {
    pdl_enter();
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t q = vec ? 4 : 1;  // elements per item
    const uint64_t width = (a_width + b_width) / q, aw = a_width / q, bw = b_width / q;
    const uint64_t items = rows * heads * width;
    for (uint64_t i = tid; i < items; i += stride) {
        const uint64_t rh = i / width, j = i % width;  // rh = row * heads + head
        const uint64_t row = rh / heads, head = rh % heads;
        if (vec) {
            reinterpret_cast<float4*>(out)[i] =
                j < aw ? reinterpret_cast<const float4*>(a)[rh * aw + j]
                       : reinterpret_cast<const float4*>(b)[(row * b_heads + (b_heads == 1 ? 0 : head)) * bw + (j - aw)];
        } else {
            out[i] = j < aw ? a[rh * aw + j] : b[(row * b_heads + (b_heads == 1 ? 0 : head)) * bw + (j - aw)];
        }
    }
}

// batched-matmul (src/kernels.cu:6296-6365): out [rows, groups * n], group g of row r being
// a[r, g k .. (g + 1) k] times b[g k .. (g + 1) k, :], or with transpose_b times
// b[g n .. (g + 1) n, :] transposed.  Sums in index order: a thread per output (consecutive
// threads read consecutive columns of b) without the transpose; with it, a warp per output
// whose lanes take every 32nd index and add their sums with a butterfly.
__global__ void __launch_bounds__(kThreads) batched_matmul_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                                                  float* __restrict__ out, uint64_t rows,
                                                                  uint64_t groups, uint64_t k, uint64_t n) {
    pdl_enter();
    const uint64_t width = groups * n, total = rows * width;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
        const uint64_t r = idx / width, col = idx % width, g = col / n, j = col % n;
        const float* in = a + r * groups * k + g * k;
        const float* w = b + g * k * n + j;
        float sum = 0.0f;
        for (uint64_t i = 0; i < k; i++) sum += in[i] * w[i * n];
        out[idx] = sum;
    }
}

__global__ void __launch_bounds__(kThreads) batched_matmul_t_kernel(const float* __restrict__ a,
                                                                    const float* __restrict__ b,
                                                                    float* __restrict__ out, uint64_t rows,
                                                                    uint64_t groups, uint64_t k, uint64_t n) {
    pdl_enter();
    const uint64_t width = groups * n, total = rows * width;
    const int lane = threadIdx.x & 31;
    const uint64_t warps = (uint64_t)gridDim.x * (kThreads / 32);
    for (uint64_t idx = (uint64_t)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5); idx < total; idx += warps) {
        const uint64_t r = idx / width, col = idx % width, g = col / n, j = col % n;
        const float* in = a + r * groups * k + g * k;
        const float* w = b + (g * n + j) * k;
        float sum = 0.0f;
        for (uint64_t i = lane; i < k; i += 32) sum += in[i] * w[i];
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) out[idx] = sum;
    }
}

__global__ void set_u64_kernel(uint64_t* dst, uint64_t value) {
    pdl_enter();
    *dst = value;
}

__global__ void __launch_bounds__(kThreads) zero_kernel(uint4* __restrict__ p, uint64_t n16) {
    pdl_enter();
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += stride)
        p[i] = make_uint4(0, 0, 0, 0);
}

}  // namespace

namespace k {

static inline unsigned vec_grid(const Device* d, uint64_t n, int vec, int lanes) {
    return grid_for(d, vec ? (n / lanes + kUnroll - 1) / kUnroll : n);
}

mg_status add(Device* d, const float* a, const float* b, float* out, uint64_t n) {
    int vec = aligned16(a) && aligned16(b) && aligned16(out);
    enqueue(d, binary_kernel<AddOp>, vec_grid(d, n, vec, 4), kThreads, 0, a, b, out, n, vec, AddOp{});
    return launched(d, "add kernel launch");
}

mg_status mul(Device* d, const float* a, const float* b, float* out, uint64_t n) {
    int vec = aligned16(a) && aligned16(b) && aligned16(out);
    enqueue(d, binary_kernel<MulOp>, vec_grid(d, n, vec, 4), kThreads, 0, a, b, out, n, vec, MulOp{});
    return launched(d, "mul kernel launch");
}

mg_status silu_mul(Device* d, const float* g, const float* u, float* out, uint64_t n) {
    int vec = aligned16(g) && aligned16(u) && aligned16(out);
    enqueue(d, binary_kernel<SiluMulOp>, vec_grid(d, n, vec, 4), kThreads, 0, g, u, out, n, vec, SiluMulOp{});
    return launched(d, "silu-mul kernel launch");
}

mg_status silu(Device* d, const float* x, float* out, uint64_t n) {
    int vec = aligned16(x) && aligned16(out);
    enqueue(d, unary_kernel<SiluOp>, vec_grid(d, n, vec, 4), kThreads, 0, x, out, n, vec, SiluOp{});
    return launched(d, "silu kernel launch");
}

mg_status scale(Device* d, const float* x, float* out, float factor, uint64_t n) {
    int vec = aligned16(x) && aligned16(out);
    enqueue(d, unary_kernel<ScaleOp>, vec_grid(d, n, vec, 4), kThreads, 0, x, out, n, vec, ScaleOp{factor});
    return launched(d, "scale kernel launch");
}

mg_status gelu_tanh(Device* d, const float* x, float* out, uint64_t n) {
    int vec = aligned16(x) && aligned16(out);
    enqueue(d, unary_kernel<GeluTanhOp>, vec_grid(d, n, vec, 4), kThreads, 0, x, out, n, vec, GeluTanhOp{});
    return launched(d, "gelu kernel launch");
}

mg_status sigmoid(Device* d, const float* x, float* out, uint64_t n) {
    int vec = aligned16(x) && aligned16(out);
    enqueue(d, unary_kernel<SigmoidOp>, vec_grid(d, n, vec, 4), kThreads, 0, x, out, n, vec, SigmoidOp{});
    return launched(d, "sigmoid kernel launch");
}

mg_status softcap(Device* d, const float* x, float* out, float cap, uint64_t n) {
    int vec = aligned16(x) && aligned16(out);
    enqueue(d, unary_kernel<SoftcapOp>, vec_grid(d, n, vec, 4), kThreads, 0, x, out, n, vec, SoftcapOp{cap});
    return launched(d, "softcap kernel launch");
}

mg_status row_scale(Device* d, const float* x, const float* scale, float* out, uint64_t rows, uint64_t cols) {
    const int vec = cols % 4 == 0 && aligned16(x) && aligned16(out);
    enqueue(d, row_scale_kernel, grid_for(d, vec ? rows * cols / 4 : rows * cols), kThreads, 0, x, scale, out, rows, cols,
            vec);
    return launched(d, "row-scale kernel launch");
}

mg_status concat_heads(Device* d, const float* a, const float* b, float* out, uint64_t rows, uint64_t heads,
                       uint64_t a_width, uint64_t b_width, uint64_t b_heads) {
    const int vec = a_width % 4 == 0 && b_width % 4 == 0 && aligned16(a) && aligned16(b) && aligned16(out);
    const uint64_t items = rows * heads * (a_width + b_width) / (vec ? 4 : 1);
    enqueue(d, concat_heads_kernel, grid_for(d, items), kThreads, 0, a, b, out, rows, heads, a_width, b_width, b_heads,
            vec);
    return launched(d, "concat kernel launch");
}

mg_status batched_matmul(Device* d, const float* a, const float* b, float* out, uint64_t rows, uint64_t groups,
                         uint64_t k, uint64_t n, int transpose_b) {
    const uint64_t total = rows * groups * n;
    if (total == 0) return MG_OK;
    if (transpose_b)
        enqueue(d, batched_matmul_t_kernel, grid_for(d, total * 32), kThreads, 0, a, b, out, rows, groups, k, n);
    else
        enqueue(d, batched_matmul_kernel, grid_for(d, total), kThreads, 0, a, b, out, rows, groups, k, n);
    return launched(d, "batched-matmul kernel launch");
}

mg_status bias_add(Device* d, const float* a, const float* bias, float* out, uint64_t cols, uint64_t n) {
    const uint64_t rows = cols ? n / cols : 0;
    int vec = (cols % 4 == 0) && aligned16(a) && aligned16(bias) && aligned16(out);
    enqueue(d, bias_add_kernel, grid_for(d, vec ? n / 4 : n), kThreads, 0, a, bias, out, cols, rows, vec);
    return launched(d, "bias-add kernel launch");
}

mg_status mul_scalar(Device* d, const float* a, const float* b, float* out, uint64_t n) {
    int vec = aligned16(a) && aligned16(out);
    enqueue(d, mul_scalar_kernel, grid_for(d, vec ? n / 4 : n), kThreads, 0, a, b, out, n, vec);
    return launched(d, "mul-scalar kernel launch");
}

mg_status half_binary(Device* d, const uint16_t* a, const uint16_t* b, uint16_t* out, uint64_t n, mg_dtype dtype,
                      int op) {
    int vec = aligned16(a) && aligned16(b) && aligned16(out);
    unsigned grid = vec_grid(d, n, vec, 8);
    if (dtype == MG_F16) {
        if (op == 0) enqueue(d, half_binary_kernel<MG_F16, 0>, grid, kThreads, 0, a, b, out, n, vec);
        else enqueue(d, half_binary_kernel<MG_F16, 1>, grid, kThreads, 0, a, b, out, n, vec);
    } else {
        if (op == 0) enqueue(d, half_binary_kernel<MG_BF16, 0>, grid, kThreads, 0, a, b, out, n, vec);
        else enqueue(d, half_binary_kernel<MG_BF16, 1>, grid, kThreads, 0, a, b, out, n, vec);
    }
    return launched(d, "half kernel launch");
}

mg_status half_binary_f32(Device* d, const float* a, const float* b, float* out, uint64_t n, mg_dtype dtype, int op) {
    int vec = aligned16(a) && aligned16(b) && aligned16(out);
    unsigned grid = vec_grid(d, n, vec, 4);
    if (dtype == MG_F16) {
        if (op == 0) enqueue(d, binary_kernel<HalfRoundTripOp<MG_F16, 0>>, grid, kThreads, 0, a, b, out, n, vec, HalfRoundTripOp<MG_F16, 0>{});
        else enqueue(d, binary_kernel<HalfRoundTripOp<MG_F16, 1>>, grid, kThreads, 0, a, b, out, n, vec, HalfRoundTripOp<MG_F16, 1>{});
    } else {
        if (op == 0) enqueue(d, binary_kernel<HalfRoundTripOp<MG_BF16, 0>>, grid, kThreads, 0, a, b, out, n, vec, HalfRoundTripOp<MG_BF16, 0>{});
        else enqueue(d, binary_kernel<HalfRoundTripOp<MG_BF16, 1>>, grid, kThreads, 0, a, b, out, n, vec, HalfRoundTripOp<MG_BF16, 1>{});
    }
    return launched(d, "half round-trip kernel launch");
}

mg_status encode_half(Device* d, const float* in, uint16_t* out, uint64_t n, mg_dtype dtype) {
    if (dtype == MG_F16) enqueue(d, encode_kernel<MG_F16>, grid_for(d, n), kThreads, 0, in, out, n);
    else enqueue(d, encode_kernel<MG_BF16>, grid_for(d, n), kThreads, 0, in, out, n);
    return launched(d, "half encode kernel launch");
}

mg_status decode_half(Device* d, const uint16_t* in, float* out, uint64_t n, mg_dtype dtype) {
    if (dtype == MG_F16) enqueue(d, decode_kernel<MG_F16>, grid_for(d, n), kThreads, 0, in, out, n);
    else enqueue(d, decode_kernel<MG_BF16>, grid_for(d, n), kThreads, 0, in, out, n);
    return launched(d, "half decode kernel launch");
}

mg_status kv_write(Device* d, const KvWriteArgs& a) {
    const uint64_t n = a.count * a.width;
    if (n == 0) return MG_OK;
    const int vec = a.width % 4 == 0 && (reinterpret_cast<uintptr_t>(a.rows) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(a.store) & 15) == 0;
    enqueue(d, kv_write_kernel, grid_for(d, vec ? n / 4 : n), kThreads, 0, a.rows, a.store, n, a.width, a.row_offset,
            a.step, vec);
    return launched(d, "kv-write kernel launch");
}

mg_status set_step_offset(Device* d, uint64_t* dst, uint64_t value) {
    enqueue(d, set_u64_kernel, 1, 1, 0, dst, value);
    return launched(d, "step offset launch");
}

mg_status fill_zero(Device* d, void* ptr, uint64_t bytes) {
    if ((reinterpret_cast<uintptr_t>(ptr) & 15) == 0 && bytes % 16 == 0) {
        if (bytes) enqueue(d, zero_kernel, grid_for(d, bytes / 16), kThreads, 0, (uint4*)ptr, bytes / 16);
        return launched(d, "zero kernel launch");
    }
    MG_CUDA(cudaMemsetAsync(ptr, 0, bytes, d->stream), "zeroing a buffer");
    return MG_OK;
}

}  // namespace k
}  // namespace mg
