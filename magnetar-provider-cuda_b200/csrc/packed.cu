// Q8_0 packed weights (`execute-direct-quantized-weights`, src/kernels.rs:309-330, 1725-1838,
// 1964-2010; src/kernels.cu:230-330): a weight stored as the checkpoint stored it, 34-byte
// blocks of one little-endian f16 scale and 32 signed 8-bit quants, unpacked once on the device
// into the quants (stored row-major, contiguous) and one f32 scale per block (the f16 widened
// exactly).  The few-row matmul streams the quants -- 1.125 bytes per weight value with the
// scales -- against f32 activations; everything else reads the dequantized values q * d.
//
// The few-row kernel: a CTA owns 256 output columns (one per thread: a transposed-storage weight
// keeps each output column's k quants contiguous) and one slice of k.  A producer lane streams
// per stage, with TMA, the [256 columns x 128 k] quants (one 128-byte row per column, 128-byte
// swizzle so that 32 threads reading their own rows hit distinct banks), the matching [256 x 4]
// scales and [M x 128] of A; each thread widens its 128 quants to f32 exactly (byte permute into
// the mantissa of 2^23 and one subtraction), multiplies them by every row of A (A read from shared
// memory as a broadcast) and adds each 32-value block's sum times the block's scale.  The slices'
// partials go to a workspace; the last CTA of a column tile adds them in slice order and applies
// bias / residual / SwiGLU (deterministic).
#include <cuda.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "internal.h"
#include "sm100.cuh"

namespace mg {
namespace {

constexpr int kQ8Block = 32;       // quants per block
constexpr int kQ8BlockBytes = 34;  // f16 scale + 32 quants
constexpr int kQCols = 256;        // output columns per CTA, one per compute thread
constexpr int kQChunk = 128;       // k per stage: four blocks, one 128-byte swizzled row per column
constexpr int kQStages = 3;
constexpr int kQMaxSplits = 64;
constexpr uint64_t kQMaxTiles = 1u << 16;  // Device::counters entries

// One thread per block: the scale widened to f32 (exact) and the 32 quants stored contiguous.
__global__ void __launch_bounds__(256) q8_unpack_kernel(const uint8_t* __restrict__ blocks, int8_t* __restrict__ quants,
                                                        float* __restrict__ scales, uint64_t nblocks) {
    pdl_enter();
    for (uint64_t b = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; b < nblocks; b += (uint64_t)gridDim.x * blockDim.x) {
        const uint16_t* src = reinterpret_cast<const uint16_t*>(blocks + b * kQ8BlockBytes);  // 2-byte aligned
        scales[b] = __half2float(__ushort_as_half(src[0]));
        uint32_t w[8];
#pragma unroll
        for (int i = 0; i < 8; i++) w[i] = (uint32_t)src[1 + 2 * i] | ((uint32_t)src[2 + 2 * i] << 16);
        uint4* dst = reinterpret_cast<uint4*>(quants + b * kQ8Block);
        dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
        dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
    }
}

// out = q * d in stored order, 16 values per thread and step (src/kernels.cu:230-246).
__global__ void __launch_bounds__(256) q8_dequantize_kernel(const int8_t* __restrict__ quants, const float* __restrict__ scales,
                                                            float* __restrict__ out, uint64_t groups) {
    pdl_enter();
    for (uint64_t g = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; g < groups; g += (uint64_t)gridDim.x * blockDim.x) {
        const uint4 q = reinterpret_cast<const uint4*>(quants)[g];
        const float d = scales[g >> 1];  // two 16-value groups per block
        const int8_t* b = reinterpret_cast<const int8_t*>(&q);
        float4* o = reinterpret_cast<float4*>(out) + 4 * g;
#pragma unroll
        for (int j = 0; j < 4; j++)
            o[j] = make_float4((float)b[4 * j] * d, (float)b[4 * j + 1] * d, (float)b[4 * j + 2] * d, (float)b[4 * j + 3] * d);
    }
}

// The logical matrix of a transposed-storage weight: out[c, r] = q[r, c] * d, through 32 x 32
// tiles so that both the quants and the output are read and written along rows.
__global__ void __launch_bounds__(256) q8_dequantize_transpose_kernel(const int8_t* __restrict__ quants,
                                                                      const float* __restrict__ scales, float* __restrict__ out,
                                                                      uint64_t stored_rows, uint64_t stored_cols) {
    pdl_enter();
    __shared__ float tile[32][33];
    const uint64_t r0 = (uint64_t)blockIdx.y * 32, c0 = (uint64_t)blockIdx.x * 32;  // stored_cols % 32 == 0
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    for (int i = ty; i < 32; i += 8) {
        const uint64_t r = r0 + i;
        if (r < stored_rows) {
            const uint64_t idx = r * stored_cols + c0 + tx;
            tile[i][tx] = (float)quants[idx] * scales[idx >> 5];
        }
    }
    __syncthreads();
    for (int i = ty; i < 32; i += 8) {
        const uint64_t r = r0 + tx;
        if (r < stored_rows) out[(c0 + i) * stored_rows + r] = tile[tx][i];
    }
}

// Embedding rows of a packed table stored untransposed: row id of the logical [vocab, dim]
// table, dequantized, times the optional scale (src/kernels.rs:3833-3997 on a packed table).
__global__ void __launch_bounds__(256) q8_embedding_kernel(const int8_t* __restrict__ quants, const float* __restrict__ scales,
                                                           const float* __restrict__ ids, float* __restrict__ out, uint64_t dim,
                                                           uint64_t num_ids, uint64_t vocab, int* flag, int has_scale, float scale) {
    pdl_enter();
    const int lane = threadIdx.x & 31;
    const uint64_t warps = (uint64_t)gridDim.x * (blockDim.x >> 5);
    for (uint64_t t = (uint64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < num_ids; t += warps) {
        const float f = ids[t];
        // the id rule of the f32 lookup: a non-negative integer below the vocabulary
        if (f < 0.0f || f != floorf(f) || !(f < (float)vocab && (uint64_t)f < vocab)) {
            if (lane == 0) atomicExch(flag, 1);
            continue;
        }
        const uint64_t id = (uint64_t)f;
        const int8_t* q = quants + id * dim;
        const float* s = scales + id * (dim / kQ8Block);
        float* o = out + t * dim;
        for (uint64_t j = lane; j < dim; j += 32) {
            float v = (float)q[j] * s[j / kQ8Block];
            if (has_scale) v *= scale;
            o[j] = v;
        }
    }
}

// Four quants (one 32-bit word) widened to f32 exactly: each byte, offset by 128 to unsigned,
// becomes the low mantissa byte of 2^23 (byte permute) and the sum 2^23 + 128 is subtracted.
__device__ __forceinline__ void q8_widen4(uint32_t w, float& a, float& b, float& c, float& d) {
    const uint32_t u = w ^ 0x80808080u;
    constexpr float kBias = 8388736.0f;  // 2^23 + 128
    a = __uint_as_float(__byte_perm(u, 0x4B00u, 0x5440u)) - kBias;
    b = __uint_as_float(__byte_perm(u, 0x4B00u, 0x5441u)) - kBias;
    c = __uint_as_float(__byte_perm(u, 0x4B00u, 0x5442u)) - kBias;
    d = __uint_as_float(__byte_perm(u, 0x4B00u, 0x5443u)) - kBias;
}

struct Q8GemvArgs {
    float* partial;  // [terms][splits][m][n]
    float* out;
    const float* addend;
    int addend_mode;  // 0 none, 1 row [n], 2 full [m, n]
    int terms;        // 1, or 2 for gated (gate: z = 0, up: z = 1)
    uint64_t m, n, k, slice_len;  // slice_len a multiple of kQChunk
    int* error;
    unsigned int* counters;  // per column tile; zero between calls (the last CTA resets it)
};

template <int M>
struct Q8Shape {
    static constexpr int kQ = kQCols * kQChunk;                      // 32 KB of quants
    static constexpr int kS = kQCols * (kQChunk / kQ8Block) * 4;     // 4 KB of scales, [256][4]
    static constexpr int kA = M * kQChunk * 4;                       // [M][128] of A
    static constexpr int kStage = (kQ + kS + kA + 1023) / 1024 * 1024;  // quants stay 1024-aligned (swizzle atom)
    static constexpr int kThreads = kQCols + 32;                     // 8 compute warps + the producer
    static constexpr int kSmem = 1024 + kQStages * kStage + 16 * kQStages;
};

template <int M>
__global__ void __launch_bounds__(Q8Shape<M>::kThreads) q8_gemv_kernel(const __grid_constant__ CUtensorMap map_a,
                                                                      const __grid_constant__ CUtensorMap map_q,
                                                                      const __grid_constant__ CUtensorMap map_s,
                                                                      const __grid_constant__ CUtensorMap map_q2,
                                                                      const __grid_constant__ CUtensorMap map_s2,
                                                                      Q8GemvArgs p) {
    using namespace sm100;
    using S = Q8Shape<M>;
    extern __shared__ uint8_t smem_raw[];
    __shared__ unsigned int s_last;
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* base_ptr = smem_raw + (base - raw);
    const uint32_t bar0 = base + kQStages * S::kStage;
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (kQStages + s); };
    const int tid = threadIdx.x, warp = tid >> 5;
    const uint64_t col0 = (uint64_t)blockIdx.x * kQCols;
    const uint64_t k0 = (uint64_t)blockIdx.y * p.slice_len;
    const uint64_t k1 = min(p.k, k0 + p.slice_len);
    const int chunks = k1 > k0 ? (int)((k1 - k0) / kQChunk) : 0;
    const CUtensorMap* mq = blockIdx.z ? &map_q2 : &map_q;
    const CUtensorMap* ms = blockIdx.z ? &map_s2 : &map_s;

    if (tid == 0) {
        for (int s = 0; s < kQStages; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), kQCols / 32);
        }
        fence_barrier_init();
        // The packed weight is written only by an upload: its first stages load before the
        // dependency wait.
        for (int c = 0; c < min(chunks, kQStages); c++) {
            const uint32_t st = base + (uint32_t)(c * S::kStage);
            const int kk = (int)(k0 + (uint64_t)c * kQChunk);
            mbar_arrive_expect_tx(full_bar(c), (uint32_t)(S::kQ + S::kS + S::kA));
            tma_load_2d(st, mq, full_bar(c), kk, (int)col0);
            tma_load_2d(st + S::kQ, ms, full_bar(c), kk / kQ8Block, (int)col0);
        }
    }
    pdl_enter();
    __syncthreads();

    float acc[M];
#pragma unroll
    for (int r = 0; r < M; r++) acc[r] = 0.0f;
    if (warp == kQCols / 32) {
        // ---- producer ----------------------------------------------------------------------
        if ((tid & 31) == 0) {
            for (int c = 0; c < chunks; c++) {
                const int s = c % kQStages;
                const uint32_t st = base + (uint32_t)(s * S::kStage);
                const int kk = (int)(k0 + (uint64_t)c * kQChunk);
                if (c >= kQStages) {
                    if (!mbar_wait(empty_bar(s), (uint32_t)(c / kQStages - 1) & 1u)) {
                        atomicExch(p.error, 1);
                        break;
                    }
                    mbar_arrive_expect_tx(full_bar(s), (uint32_t)(S::kQ + S::kS + S::kA));
                    tma_load_2d(st, mq, full_bar(s), kk, (int)col0);
                    tma_load_2d(st + S::kQ, ms, full_bar(s), kk / kQ8Block, (int)col0);
                }
                tma_load_2d(st + S::kQ + S::kS, &map_a, full_bar(s), kk, 0);
            }
        }
        __syncwarp();
    } else {
        // ---- compute: thread tid owns output column col0 + tid --------------------------------
        const uint32_t sw = (uint32_t)(tid & 7);  // the 128-byte swizzle's chunk permutation for this row
        for (int c = 0; c < chunks; c++) {
            const int s = c % kQStages;
            if (!mbar_wait(full_bar(s), (uint32_t)(c / kQStages) & 1u)) {
                atomicExch(p.error, 1);
                break;
            }
            const uint8_t* st = base_ptr + s * S::kStage;
            const uint8_t* qrow = st + tid * kQChunk;
            const float4 sc = *reinterpret_cast<const float4*>(st + S::kQ + tid * 16);
            const float* a_s = reinterpret_cast<const float*>(st + S::kQ + S::kS);  // [M][128]
            const float scl[4] = {sc.x, sc.y, sc.z, sc.w};
#pragma unroll
            for (int blk = 0; blk < 4; blk++) {
                const uint4 q0 = *reinterpret_cast<const uint4*>(qrow + (((2u * blk) ^ sw) << 4));
                const uint4 q1 = *reinterpret_cast<const uint4*>(qrow + (((2u * blk + 1u) ^ sw) << 4));
                float f[32];
                q8_widen4(q0.x, f[0], f[1], f[2], f[3]);
                q8_widen4(q0.y, f[4], f[5], f[6], f[7]);
                q8_widen4(q0.z, f[8], f[9], f[10], f[11]);
                q8_widen4(q0.w, f[12], f[13], f[14], f[15]);
                q8_widen4(q1.x, f[16], f[17], f[18], f[19]);
                q8_widen4(q1.y, f[20], f[21], f[22], f[23]);
                q8_widen4(q1.z, f[24], f[25], f[26], f[27]);
                q8_widen4(q1.w, f[28], f[29], f[30], f[31]);
#pragma unroll
                for (int r = 0; r < M; r++) {
                    const float* ar = a_s + r * kQChunk + blk * kQ8Block;
                    float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
                    for (int j = 0; j < kQ8Block; j += 8) {
                        const float4 x0 = *reinterpret_cast<const float4*>(ar + j);
                        const float4 x1 = *reinterpret_cast<const float4*>(ar + j + 4);
                        s0 = fmaf(x0.x, f[j], s0);
                        s1 = fmaf(x0.y, f[j + 1], s1);
                        s0 = fmaf(x0.z, f[j + 2], s0);
                        s1 = fmaf(x0.w, f[j + 3], s1);
                        s0 = fmaf(x1.x, f[j + 4], s0);
                        s1 = fmaf(x1.y, f[j + 5], s1);
                        s0 = fmaf(x1.z, f[j + 6], s0);
                        s1 = fmaf(x1.w, f[j + 7], s1);
                    }
                    acc[r] = fmaf(scl[blk], s0 + s1, acc[r]);
                }
            }
            __syncwarp();
            if ((tid & 31) == 0) mbar_arrive(empty_bar(s));
        }
        // this slice's partial, one coalesced row per output row
        const uint64_t col = col0 + tid;
        if (col < p.n) {
            float* part = p.partial + ((uint64_t)blockIdx.z * gridDim.y + blockIdx.y) * p.m * p.n;
#pragma unroll
            for (int r = 0; r < M; r++)
                if ((uint64_t)r < p.m) part[(uint64_t)r * p.n + col] = acc[r];
        }
    }
    // ---- the last CTA of this column tile (over slices and gate / up) finishes it --------------
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(&p.counters[blockIdx.x], 1u) == gridDim.y * gridDim.z - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (tid < kQCols) {
        const uint64_t col = col0 + tid;
        const int splits = (int)gridDim.y;
        const uint64_t mn = p.m * p.n;
        if (col < p.n) {
            for (uint64_t r = 0; r < p.m; r++) {
                const uint64_t off = r * p.n + col;
                float g = 0.0f;
                for (int sl = 0; sl < splits; sl++) g += __ldcg(p.partial + (uint64_t)sl * mn + off);
                float v;
                if (p.terms == 2) {
                    float u = 0.0f;
                    for (int sl = 0; sl < splits; sl++) u += __ldcg(p.partial + ((uint64_t)splits + sl) * mn + off);
                    v = (g * (1.0f / (1.0f + expf(-g)))) * u;
                } else {
                    v = g;
                    if (p.addend_mode == 1) v += p.addend[col];
                    else if (p.addend_mode == 2) v += p.addend[off];
                }
                p.out[off] = v;
            }
        }
    }
    if (tid == 0) p.counters[blockIdx.x] = 0u;
}

PFN_cuTensorMapEncodeTiled_v12000 q8_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

mg_status q8_map(CUtensorMap* map, CUtensorMapDataType type, void* ptr, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                 uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
    auto fn = q8_encode_fn();
    if (!fn) return fail(MG_DRIVER_FAILED, "the driver does not provide cuTensorMapEncodeTiled");
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, type, 2, ptr, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(MG_DRIVER_FAILED, "encoding a TMA descriptor failed (CUresult %d)", (int)r);
    return MG_OK;
}

template <int M>
mg_status launch_q8_gemv(Device* d, dim3 grid, const CUtensorMap* maps, const Q8GemvArgs& p) {
    using S = Q8Shape<M>;
    static bool configured[64] = {false};
    if (!configured[d->ordinal & 63]) {
        MG_CUDA(cudaFuncSetAttribute(q8_gemv_kernel<M>, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmem),
                "configuring the packed gemv kernel");
        configured[d->ordinal & 63] = true;
    }
    enqueue(d, q8_gemv_kernel<M>, grid, S::kThreads, S::kSmem, maps[0], maps[1], maps[2], maps[3], maps[4], p);
    return launched(d, "packed gemv launch");
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; }

}  // namespace

namespace k {

mg_status q8_unpack(Device* d, const uint8_t* blocks, int8_t* quants, float* scales, uint64_t nblocks) {
    uint64_t grid = (nblocks + 255) / 256;
    if (grid > (uint64_t)d->sm_count * 8) grid = (uint64_t)d->sm_count * 8;
    enqueue(d, q8_unpack_kernel, (unsigned)(grid ? grid : 1), 256, 0, blocks, quants, scales, nblocks);
    return launched(d, "packed weight unpack launch");
}

mg_status q8_dequantize(Device* d, const Buffer* b, float* out, bool stored_order) {
    const int8_t* q = static_cast<const int8_t*>(b->ptr);
    if (stored_order || !b->q8_transposed) {
        const uint64_t groups = b->q8_rows * b->q8_cols / 16;
        uint64_t grid = (groups + 255) / 256;
        if (grid > (uint64_t)d->sm_count * 8) grid = (uint64_t)d->sm_count * 8;
        enqueue(d, q8_dequantize_kernel, (unsigned)(grid ? grid : 1), 256, 0, q, (const float*)b->q8_scales, out, groups);
        return launched(d, "packed weight dequantize launch");
    }
    if ((b->q8_rows + 31) / 32 > 65535) return fail(MG_SHAPE_UNSUPPORTED, "packed weight has too many stored rows");
    dim3 grid((unsigned)(b->q8_cols / 32), (unsigned)((b->q8_rows + 31) / 32));
    enqueue(d, q8_dequantize_transpose_kernel, grid, 256, 0, q, (const float*)b->q8_scales, out, b->q8_rows, b->q8_cols);
    return launched(d, "packed weight dequantize launch");
}

mg_status q8_embedding(Device* d, const Buffer* table, const float* ids, float* out, uint64_t num_ids, int* flag,
                       int has_scale, float scale) {
    uint64_t grid = (num_ids + 7) / 8;
    if (grid > (uint64_t)d->sm_count * 8) grid = (uint64_t)d->sm_count * 8;
    enqueue(d, q8_embedding_kernel, (unsigned)(grid ? grid : 1), 256, 0, (const int8_t*)table->ptr,
            (const float*)table->q8_scales, ids, out, table->q8_cols, num_ids, table->q8_rows, flag, has_scale, scale);
    return launched(d, "packed embedding launch");
}

// The few-row kernel takes a matmul when every B is a transposed-storage packed weight, A is
// contiguous and 16-byte aligned, M <= 16 and k is a multiple of 128 (the scales' rows then
// stay 16-byte multiples for TMA).
bool q8_gemv_eligible(const GemmArgs& g) {
    const int terms = g.gated ? 2 : 1;
    for (int t = 0; t < terms; t++)
        if (!g.packed[t] || !g.packed[t]->q8_transposed) return false;
    return g.m >= 1 && g.m <= 16 && !g.transpose_a && !g.transpose_b && g.k % kQChunk == 0 && aligned16(g.a) &&
           (g.n + kQCols - 1) / kQCols <= kQMaxTiles && g.k < (1ull << 31) && g.n < (1ull << 31);
}

mg_status q8_gemv(Device* d, const GemmArgs& g) {
    const uint64_t tiles = (g.n + kQCols - 1) / kQCols;
    const int terms = g.gated ? 2 : 1;
    const int mp = g.m <= 1 ? 1 : g.m <= 2 ? 2 : g.m <= 4 ? 4 : g.m <= 8 ? 8 : 16;
    // k slices for about two CTAs per SM (one at the larger row counts)
    const uint64_t per_sm = mp <= 1 ? 2 : 1;
    const uint64_t chunks = g.k / kQChunk;
    uint64_t splits = ((uint64_t)d->sm_count * per_sm + tiles * terms - 1) / (tiles * terms);
    if (splits > chunks) splits = chunks;
    if (splits > (uint64_t)kQMaxSplits) splits = kQMaxSplits;
    if (splits < 1) splits = 1;
    Q8GemvArgs p;
    p.slice_len = (chunks + splits - 1) / splits * kQChunk;
    splits = (g.k + p.slice_len - 1) / p.slice_len;
    p.out = g.out;
    p.addend = g.addend;
    p.addend_mode = g.addend_mode;
    p.terms = terms;
    p.m = g.m;
    p.n = g.n;
    p.k = g.k;
    p.error = d->flags + 2;
    p.counters = d->counters;
    MG_TRY(scratch(d, 0, (size_t)terms * splits * g.m * g.n * sizeof(float), (void**)&p.partial));
    CUtensorMap maps[5];
    MG_TRY(q8_map(&maps[0], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, const_cast<float*>(g.a), g.k, g.m, g.k * 4, kQChunk,
                  (uint32_t)mp, CU_TENSOR_MAP_SWIZZLE_NONE));
    for (int t = 0; t < 2; t++) {
        const Buffer* w = g.packed[t < terms ? t : 0];
        MG_TRY(q8_map(&maps[1 + 2 * t], CU_TENSOR_MAP_DATA_TYPE_UINT8, w->ptr, g.k, g.n, g.k, kQChunk, kQCols,
                      CU_TENSOR_MAP_SWIZZLE_128B));
        MG_TRY(q8_map(&maps[2 + 2 * t], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, w->q8_scales, g.k / kQ8Block, g.n,
                      g.k / kQ8Block * 4, kQChunk / kQ8Block, kQCols, CU_TENSOR_MAP_SWIZZLE_NONE));
    }
    dim3 grid((unsigned)tiles, (unsigned)splits, (unsigned)terms);
    switch (mp) {
        case 1: return launch_q8_gemv<1>(d, grid, maps, p);
        case 2: return launch_q8_gemv<2>(d, grid, maps, p);
        case 4: return launch_q8_gemv<4>(d, grid, maps, p);
        case 8: return launch_q8_gemv<8>(d, grid, maps, p);
        default: return launch_q8_gemv<16>(d, grid, maps, p);
    }
}

// A matmul with packed B (src/kernels.rs:5581-5600): the few-row kernel when eligible, else each
// packed weight dequantized (stored order) for the duration of the call and the f32 matmul.
mg_status q8_matmul(Device* d, const GemmArgs& g) {
    if (q8_gemv_eligible(g)) return q8_gemv(d, g);
    GemmArgs f = g;
    void* mem[2] = {nullptr, nullptr};
    mg_status s = MG_OK;
    for (int t = 0; t < 2 && s == MG_OK; t++) {
        const Buffer* w = g.packed[t];
        if (!w) continue;
        s = device_alloc(d, w->q8_rows * w->q8_cols * sizeof(float), &mem[t]);
        if (s == MG_OK) s = q8_dequantize(d, w, static_cast<float*>(mem[t]), true);
        (t == 0 ? f.b : f.b2) = static_cast<const float*>(mem[t]);
        f.packed[t] = nullptr;
    }
    if (s == MG_OK) {
        // the stored matrix is the logical B, or its transpose for a transposed-storage weight;
        // a gated pair with one packed and one f32 weight is dequantized only when both agree
        const Buffer* w = g.packed[0] ? g.packed[0] : g.packed[1];
        const bool flip = w->q8_transposed != 0;
        if (g.gated && g.packed[0] && g.packed[1] && g.packed[0]->q8_transposed != g.packed[1]->q8_transposed)
            s = fail(MG_LAYOUT_UNSUPPORTED, "gated-matmul's packed weights differ in storage order");
        else if (g.gated && flip && (!g.packed[0] || !g.packed[1]))
            s = fail(MG_LAYOUT_UNSUPPORTED, "gated-matmul mixes a transposed-storage packed weight with an f32 weight");
        if (s == MG_OK) {
            if (flip) f.transpose_b = !g.transpose_b;
            f.b_prep[0] = f.b_prep[1] = nullptr;
            f.b16[0] = f.b16[1] = nullptr;
            f.b_stable = 0;
            s = gemm(d, f);
        }
    }
    for (int t = 0; t < 2; t++)
        if (mem[t]) device_free(d, mem[t]);
    return s;
}

}  // namespace k
}  // namespace mg
