// Q8_0 packed weights (`execute-direct-quantized-weights`, src/kernels.rs:309-330, 1725-1838,
// 1964-2010; src/kernels.cu:230-330): a weight stored as the checkpoint stored it, 34-byte
// blocks of one little-endian f16 scale and 32 signed 8-bit quants, unpacked once on the device
// into the quants (stored row-major, contiguous) and one f32 scale per block (the f16 widened
// exactly).  The few-row matmul streams the quants -- 1.125 bytes per weight value with the
// scales -- against f32 activations; everything else reads the dequantized values q * d.
//
// A transposed-storage weight (each output column's k quants contiguous) whose k is a multiple of
// 128 is unpacked into the tiled layout the few-row kernel streams: per 256 output columns and
// 128 k one 32 KB record of quants, column after column (128 bytes each, its eight 16-byte pieces
// permuted so that 32 threads reading their own columns' piece hit distinct banks), and one 4 KB
// record of the matching [256][4] scales, records in column-tile-major order.  A CTA owns one
// tile of 256 columns (one per thread) and one slice of k, i.e. one contiguous run of records: a
// producer lane moves per stage the two records with two bulk copies and [M x 128] of A with TMA;
// each thread widens its 128 quants to f32 exactly (byte permute into the mantissa of 2^23 and
// one subtraction), multiplies them by every row of A (a broadcast read of shared memory) and
// adds each 32-value block's sum times the block's scale.  The slices' partials go to a
// workspace; the last CTA of a column tile adds them in slice order and applies bias / residual /
// SwiGLU (deterministic).
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

// Where stored element (r, c) of a packed weight lives: its quant's byte offset and its scale's
// index, in the plain or the tiled layout (c a multiple of 16 addresses 16 contiguous quants).
struct Q8View {
    const int8_t* q;
    const float* s;
    uint64_t rows, cols, chunks;  // chunks = cols / 128 (tiled)
    int tiled;
};
__device__ __forceinline__ uint64_t q8_qoff(const Q8View& v, uint64_t r, uint64_t c) {
    if (!v.tiled) return r * v.cols + c;
    const uint64_t rec = (r >> 8) * v.chunks + (c >> 7);
    const uint32_t piece = (uint32_t)((c & 127) >> 4) ^ (uint32_t)(r & 7);
    return ((rec << 8) + (r & 255)) * kQChunk + (piece << 4) + (c & 15);
}
__device__ __forceinline__ uint64_t q8_soff(const Q8View& v, uint64_t r, uint64_t c) {
    if (!v.tiled) return (r * v.cols + c) >> 5;
    const uint64_t rec = (r >> 8) * v.chunks + (c >> 7);
    return ((rec << 8) + (r & 255)) * 4 + ((c & 127) >> 5);
}

// One thread per block: the scale widened to f32 (exact) and the 32 quants stored as the layout
// places them.
__global__ void __launch_bounds__(256) q8_unpack_kernel(const uint8_t* __restrict__ blocks, Q8View v, uint64_t nblocks) {
    pdl_enter();
    int8_t* quants = const_cast<int8_t*>(v.q);
    float* scales = const_cast<float*>(v.s);
    const uint64_t per_row = v.cols / kQ8Block;
    for (uint64_t b = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; b < nblocks; b += (uint64_t)gridDim.x * blockDim.x) {
        const uint16_t* src = reinterpret_cast<const uint16_t*>(blocks + b * kQ8BlockBytes);  // 2-byte aligned
        const uint64_t r = b / per_row, c = (b % per_row) * kQ8Block;
        scales[q8_soff(v, r, c)] = __half2float(__ushort_as_half(src[0]));
        uint32_t w[8];
#pragma unroll
        for (int i = 0; i < 8; i++) w[i] = (uint32_t)src[1 + 2 * i] | ((uint32_t)src[2 + 2 * i] << 16);
        *reinterpret_cast<uint4*>(quants + q8_qoff(v, r, c)) = make_uint4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<uint4*>(quants + q8_qoff(v, r, c + 16)) = make_uint4(w[4], w[5], w[6], w[7]);
    }
}

// out = q * d in stored order, 16 values per thread and step (src/kernels.cu:230-246).
__global__ void __launch_bounds__(256) q8_dequantize_kernel(Q8View v, float* __restrict__ out, uint64_t groups) {
    pdl_enter();
    const uint64_t per_row = v.cols / 16;
    for (uint64_t g = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; g < groups; g += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t r = g / per_row, c = (g % per_row) * 16;
        const uint4 q = *reinterpret_cast<const uint4*>(v.q + q8_qoff(v, r, c));
        const float d = v.s[q8_soff(v, r, c)];
        const int8_t* b = reinterpret_cast<const int8_t*>(&q);
        float4* o = reinterpret_cast<float4*>(out) + 4 * g;
#pragma unroll
        for (int j = 0; j < 4; j++)
            o[j] = make_float4((float)b[4 * j] * d, (float)b[4 * j + 1] * d, (float)b[4 * j + 2] * d, (float)b[4 * j + 3] * d);
    }
}

// The logical matrix of a transposed-storage weight: out[c, r] = q[r, c] * d, through 32 x 32
// tiles so that both the quants and the output are read and written along rows.
__global__ void __launch_bounds__(256) q8_dequantize_transpose_kernel(Q8View v, float* __restrict__ out) {
    pdl_enter();
    __shared__ float tile[32][33];
    const uint64_t r0 = (uint64_t)blockIdx.y * 32, c0 = (uint64_t)blockIdx.x * 32;  // cols % 32 == 0
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    for (int i = ty; i < 32; i += 8) {
        const uint64_t r = r0 + i;
        if (r < v.rows) tile[i][tx] = (float)v.q[q8_qoff(v, r, c0 + tx)] * v.s[q8_soff(v, r, c0 + tx)];
    }
    __syncthreads();
    for (int i = ty; i < 32; i += 8) {
        const uint64_t r = r0 + tx;
        if (r < v.rows) out[(c0 + i) * v.rows + r] = tile[tx][i];
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

// Packed pairs of f32 (Blackwell's two-lane f32 arithmetic): each lane rounds as the scalar form.
__device__ __forceinline__ uint64_t q8_pack(uint32_t lo, uint32_t hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
    return r;
}
__device__ __forceinline__ uint64_t q8_packf(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ uint64_t q8_sub2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ void q8_fma2(uint64_t& d, uint64_t a, uint64_t b) {
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(d) : "l"(a), "l"(b));
}
__device__ __forceinline__ float q8_sum2(uint64_t v) {
    float lo, hi;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
    return lo + hi;
}

// Sixteen quants (one 16-byte piece) widened to f32 exactly, as eight packed pairs: each byte,
// offset by 128 to unsigned, becomes the low mantissa byte of 2^23 (byte permute) and 2^23 + 128
// is subtracted from both lanes of a pair at once.
__device__ __forceinline__ void q8_widen16(uint4 q, uint64_t* f) {
    const uint64_t bias = q8_packf(8388736.0f, 8388736.0f);  // 2^23 + 128
    const uint32_t w[4] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u, q.z ^ 0x80808080u, q.w ^ 0x80808080u};
#pragma unroll
    for (int i = 0; i < 4; i++) {
        f[2 * i] = q8_sub2(q8_pack(__byte_perm(w[i], 0x4B00u, 0x5440u), __byte_perm(w[i], 0x4B00u, 0x5441u)), bias);
        f[2 * i + 1] = q8_sub2(q8_pack(__byte_perm(w[i], 0x4B00u, 0x5442u), __byte_perm(w[i], 0x4B00u, 0x5443u)), bias);
    }
}

constexpr int kQMaxCluster = 16;  // k slices x terms of one column tile (above 8 only where one wave holds them)

struct Q8GemvArgs {
    const int8_t* quants[2];  // tiled quants of the weight (z = 0) and, gated, the up weight (z = 1)
    const float* scales[2];
    uint64_t chunks;          // k / 128: records per column tile
    float* out;
    const float* addend;
    int addend_mode;  // 0 none, 1 row [n], 2 full [m, n]
    int terms;        // 1, or 2 for gated (gate: z = 0, up: z = 1)
    int splits;       // k slices; the cluster is (1, splits, terms)
    int band;         // floats of the flattened [m][256] partial each cluster CTA finishes (multiple of 4)
    uint64_t m, n, k, slice_len;  // slice_len a multiple of kQChunk
    int* error;
};

template <int M>
struct Q8Shape {
    static constexpr int kQ = kQCols * kQChunk;                      // 32 KB of quants
    static constexpr int kS = kQCols * (kQChunk / kQ8Block) * 4;     // 4 KB of scales, [256][4]
    static constexpr int kA = M * kQChunk * 4;                       // [M][128] of A
    static constexpr int kStage = (kQ + kS + kA + 127) / 128 * 128;
    static constexpr int kStages = M == 1 ? 3 : 2;                   // two CTAs fit an SM
    static constexpr int kPart = M * kQCols * 4;                     // this CTA's partial, in the drained ring
    static constexpr int kRecv = (M * kQCols + 4 * kQMaxCluster) * 4;  // the other CTAs' partials of this CTA's band
    static constexpr int kThreads = kQCols + 32;                     // 8 compute warps + the producer
    static_assert(kPart <= kStages * kStage, "the partial fits the drained ring");
    static constexpr int kSmem = 128 + kStages * kStage + kRecv + 8 * (2 * kStages + 1);
    static_assert(2 * (kSmem + 1024) <= 228 * 1024, "two CTAs fit an SM");
};

// The k slices of one column tile (and, gated, both terms) form a cluster: each CTA stages its
// [m][256] partial in its drained ring and sends every band of it to the CTA that owns the band
// (one bulk copy into that CTA's receive region); owners add the partials in slice order and
// apply bias / residual / SwiGLU -- deterministic, and nothing goes through global memory.
template <int M>
__global__ void __launch_bounds__(Q8Shape<M>::kThreads) q8_gemv_kernel(const __grid_constant__ CUtensorMap map_a,
                                                                      const __grid_constant__ Q8GemvArgs p) {
    using namespace sm100;
    using S = Q8Shape<M>;
    constexpr int kQStages = S::kStages;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 127u) & ~127u;
    uint8_t* base_ptr = smem_raw + (base - raw);
    const uint32_t recv = base + kQStages * S::kStage;
    const uint32_t bar0 = recv + S::kRecv;
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (kQStages + s); };
    const uint32_t recv_bar = bar0 + 8u * (2 * kQStages);
    float* partf = reinterpret_cast<float*>(base_ptr);
    const float* recvf = reinterpret_cast<const float*>(base_ptr + kQStages * S::kStage);
    const int tid = threadIdx.x, warp = tid >> 5;
    const uint64_t col0 = (uint64_t)blockIdx.x * kQCols;
    const uint64_t k0 = (uint64_t)blockIdx.y * p.slice_len;
    const uint64_t k1 = min(p.k, k0 + p.slice_len);
    const int chunks = k1 > k0 ? (int)((k1 - k0) / kQChunk) : 0;
    const int nc = p.splits * p.terms;
    const int rank = (int)blockIdx.y + p.splits * (int)blockIdx.z;  // the cluster spans y and z whole
    const int F = (int)p.m * kQCols;
    const int my_lo = min(F, rank * p.band), my_hi = min(F, my_lo + p.band);
    // this CTA's records: column tile blockIdx.x, chunks from k0 / 128 on
    const uint64_t rec0 = (uint64_t)blockIdx.x * p.chunks + k0 / kQChunk;
    const int8_t* qrec = p.quants[blockIdx.z] + rec0 * S::kQ;
    const float* srec = p.scales[blockIdx.z] + rec0 * (S::kS / 4);

    if (tid == 0) {
        for (int s = 0; s < kQStages; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), kQCols / 32);
        }
        mbar_init(recv_bar, 1);
        fence_barrier_init();
        mbar_arrive_expect_tx(recv_bar, (uint32_t)((nc - 1) * (my_hi - my_lo) * 4));
        // The packed weight is written only by an upload (which completes before it returns):
        // its first stages load before the dependency wait.
        for (int c = 0; c < min(chunks, kQStages); c++) {
            const uint32_t st = base + (uint32_t)(c * S::kStage);
            mbar_arrive_expect_tx(full_bar(c), (uint32_t)(S::kQ + S::kS + S::kA));
            bulk_load(st, qrec + (uint64_t)c * S::kQ, S::kQ, full_bar(c));
            bulk_load(st + S::kQ, srec + (uint64_t)c * (S::kS / 4), S::kS, full_bar(c));
        }
    }
    cluster_arrive();  // phase 1: every CTA's receive barrier is armed before anyone sends
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
                    bulk_load(st, qrec + (uint64_t)c * S::kQ, S::kQ, full_bar(s));
                    bulk_load(st + S::kQ, srec + (uint64_t)c * (S::kS / 4), S::kS, full_bar(s));
                }
                tma_load_2d(st + S::kQ + S::kS, &map_a, full_bar(s), kk, 0);
            }
        }
        __syncwarp();
    } else {
        // ---- compute: thread tid owns output column col0 + tid --------------------------------
        const uint32_t sw = (uint32_t)(tid & 7);  // the piece permutation of this column's record row
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
                uint64_t f[16];  // the block's 32 quants as f32 pairs
                q8_widen16(*reinterpret_cast<const uint4*>(qrow + (((2u * blk) ^ sw) << 4)), f);
                q8_widen16(*reinterpret_cast<const uint4*>(qrow + (((2u * blk + 1u) ^ sw) << 4)), f + 8);
#pragma unroll
                for (int r = 0; r < M; r++) {
                    const float* ar = a_s + r * kQChunk + blk * kQ8Block;
                    // even and odd k of the block in the two lanes, two chains per row
                    uint64_t s2a = 0ull, s2b = 0ull;
#pragma unroll
                    for (int j = 0; j < kQ8Block; j += 8) {
                        const float4 x0 = *reinterpret_cast<const float4*>(ar + j);
                        const float4 x1 = *reinterpret_cast<const float4*>(ar + j + 4);
                        q8_fma2(s2a, q8_packf(x0.x, x0.y), f[j / 2]);
                        q8_fma2(s2b, q8_packf(x0.z, x0.w), f[j / 2 + 1]);
                        q8_fma2(s2a, q8_packf(x1.x, x1.y), f[j / 2 + 2]);
                        q8_fma2(s2b, q8_packf(x1.z, x1.w), f[j / 2 + 3]);
                    }
                    acc[r] = fmaf(scl[blk], q8_sum2(s2a) + q8_sum2(s2b), acc[r]);
                }
            }
            __syncwarp();
            if ((tid & 31) == 0) mbar_arrive(empty_bar(s));
        }
    }
    // ---- this CTA's partial, [m][256] in the drained ring ----------------------------------------
    __syncthreads();
    if (tid < kQCols) {
#pragma unroll
        for (int r = 0; r < M; r++)
            if ((uint64_t)r < p.m) partf[r * kQCols + tid] = acc[r];
    }
    fence_proxy_async();  // the partial is read by bulk copies next
    __syncthreads();
    // ---- exchange: each band of the partial to the CTA that owns it ---------------------------
    cluster_wait();  // phase 1
    if (tid == 0) {
        for (int o = 0; o < nc; o++) {
            if (o == rank) continue;
            const int lo = min(F, o * p.band), hi = min(F, lo + p.band);
            if (hi > lo)
                bulk_copy_to_cluster(mapa(recv + (uint32_t)(rank * p.band * 4), (uint32_t)o), base + (uint32_t)(lo * 4),
                                     (uint32_t)((hi - lo) * 4), mapa(recv_bar, (uint32_t)o));
        }
    }
    if (!mbar_wait(recv_bar, 0)) atomicExch(p.error, 1);
    cluster_arrive();  // phase 2: every copy into this CTA has landed
    // ---- finish this CTA's band: slices in order, per term -----------------------------------
    for (int e = my_lo + tid; e < my_hi; e += blockDim.x) {
        const int r = e / kQCols, c = e % kQCols;
        const uint64_t col = col0 + c;
        if (col >= p.n) continue;
        auto from = [&](int src) { return src == rank ? partf[e] : recvf[src * p.band + (e - my_lo)]; };
        float g = 0.0f;
        for (int sl = 0; sl < p.splits; sl++) g += from(sl);
        float v;
        if (p.terms == 2) {
            float u = 0.0f;
            for (int sl = 0; sl < p.splits; sl++) u += from(p.splits + sl);
            v = (g * (1.0f / (1.0f + expf(-g)))) * u;
        } else {
            v = g;
            if (p.addend_mode == 1) v += p.addend[col];
            else if (p.addend_mode == 2) v += p.addend[(uint64_t)r * p.n + col];
        }
        p.out[(uint64_t)r * p.n + col] = v;
    }
    cluster_wait();  // phase 2: every copy out of this CTA's shared memory has landed
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
mg_status launch_q8_gemv(Device* d, dim3 grid, const CUtensorMap& map_a, const Q8GemvArgs& p) {
    using S = Q8Shape<M>;
    static bool configured[64] = {false};
    if (!configured[d->ordinal & 63]) {
        MG_CUDA(cudaFuncSetAttribute(q8_gemv_kernel<M>, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmem),
                "configuring the packed gemv kernel");
        MG_CUDA(cudaFuncSetAttribute(q8_gemv_kernel<M>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1),
                "allowing the packed gemv kernel clusters of up to 16");
        configured[d->ordinal & 63] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(S::kThreads, 1, 1);
    cfg.dynamicSmemBytes = S::kSmem;
    cfg.stream = d->stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = grid.y;
    attr[0].val.clusterDim.z = grid.z;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = d->pdl ? 2 : 1;
    MG_CUDA(cudaLaunchKernelEx(&cfg, q8_gemv_kernel<M>, map_a, p), "packed gemv launch");
    return launched(d, "packed gemv launch");
}

// Whether all `tiles` clusters of `nc` CTAs of q8_gemv_kernel<M> fit the GPU at once (the
// occupancy query, once per size and device); sizes up to 8 always launch.
template <int M>
bool q8_cluster_fits(Device* d, int nc, uint64_t tiles, int terms) {
    using S = Q8Shape<M>;
    if (nc <= 8) return true;
    static int active[64][kQMaxCluster + 1];  // clusters the GPU holds at once, + 1 (0: not asked yet)
    int& a = active[d->ordinal & 63][nc];
    if (a == 0) {
        int clusters = 0;
        cudaLaunchConfig_t q = {};
        q.gridDim = dim3(1, (unsigned)(nc / terms), (unsigned)terms);
        q.blockDim = dim3(S::kThreads, 1, 1);
        q.dynamicSmemBytes = S::kSmem;
        cudaLaunchAttribute ca;
        ca.id = cudaLaunchAttributeClusterDimension;
        ca.val.clusterDim.x = 1;
        ca.val.clusterDim.y = (unsigned)(nc / terms);
        ca.val.clusterDim.z = (unsigned)terms;
        q.attrs = &ca;
        q.numAttrs = 1;
        if (cudaFuncSetAttribute(q8_gemv_kernel<M>, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmem) != cudaSuccess ||
            cudaFuncSetAttribute(q8_gemv_kernel<M>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess ||
            cudaOccupancyMaxActiveClusters(&clusters, q8_gemv_kernel<M>, &q) != cudaSuccess) {
            (void)cudaGetLastError();
            clusters = 0;
        }
        a = clusters + 1;
    }
    return (uint64_t)(a - 1) >= tiles;
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; }

}  // namespace

namespace k {

Q8View view(const Buffer* b) {
    Q8View v;
    v.q = static_cast<const int8_t*>(b->ptr);
    v.s = b->q8_scales;
    v.rows = b->q8_rows;
    v.cols = b->q8_cols;
    v.chunks = b->q8_cols / kQChunk;
    v.tiled = b->q8_tiled;
    return v;
}

mg_status q8_unpack(Device* d, const uint8_t* blocks, const Buffer* b) {
    const uint64_t nblocks = b->q8_rows * b->q8_cols / kQ8Block;
    uint64_t grid = (nblocks + 255) / 256;
    if (grid > (uint64_t)d->sm_count * 8) grid = (uint64_t)d->sm_count * 8;
    enqueue(d, q8_unpack_kernel, (unsigned)(grid ? grid : 1), 256, 0, blocks, view(b), nblocks);
    return launched(d, "packed weight unpack launch");
}

mg_status q8_dequantize(Device* d, const Buffer* b, float* out, bool stored_order) {
    if (stored_order || !b->q8_transposed) {
        const uint64_t groups = b->q8_rows * b->q8_cols / 16;
        uint64_t grid = (groups + 255) / 256;
        if (grid > (uint64_t)d->sm_count * 8) grid = (uint64_t)d->sm_count * 8;
        enqueue(d, q8_dequantize_kernel, (unsigned)(grid ? grid : 1), 256, 0, view(b), out, groups);
        return launched(d, "packed weight dequantize launch");
    }
    if ((b->q8_rows + 31) / 32 > 65535) return fail(MG_SHAPE_UNSUPPORTED, "packed weight has too many stored rows");
    dim3 grid((unsigned)(b->q8_cols / 32), (unsigned)((b->q8_rows + 31) / 32));
    enqueue(d, q8_dequantize_transpose_kernel, grid, 256, 0, view(b), out);
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

// The few-row kernel takes a matmul when every B is a tiled packed weight (transposed storage,
// k a multiple of 128), A is contiguous and 16-byte aligned and M <= 16.
bool q8_gemv_eligible(const GemmArgs& g) {
    const int terms = g.gated ? 2 : 1;
    for (int t = 0; t < terms; t++)
        if (!g.packed[t] || !g.packed[t]->q8_tiled) return false;
    return g.m >= 1 && g.m <= 16 && !g.transpose_a && !g.transpose_b && g.k % kQChunk == 0 && aligned16(g.a) &&
           g.k < (1ull << 31) && g.n < (1ull << 31);
}

mg_status q8_gemv(Device* d, const GemmArgs& g) {
    const uint64_t tiles = (g.n + kQCols - 1) / kQCols;
    const int terms = g.gated ? 2 : 1;
    const int mp = g.m <= 1 ? 1 : g.m <= 2 ? 2 : g.m <= 4 ? 4 : g.m <= 8 ? 8 : 16;
    // k slices for about two CTAs per SM, at most a portable cluster of them per column tile
    const uint64_t chunks = g.k / kQChunk;
    uint64_t splits = ((uint64_t)d->sm_count * 2 + tiles * terms - 1) / (tiles * terms);
    if (splits > (uint64_t)(kQMaxCluster / terms)) splits = kQMaxCluster / terms;
    if (splits > chunks) splits = chunks;
    if (splits < 1) splits = 1;
    // clusters above 8 CTAs only where the GPU holds them (non-portable sizes)
    auto fits = [&](int nc) {
        switch (mp) {
            case 1: return q8_cluster_fits<1>(d, nc, tiles, terms);
            case 2: return q8_cluster_fits<2>(d, nc, tiles, terms);
            case 4: return q8_cluster_fits<4>(d, nc, tiles, terms);
            case 8: return q8_cluster_fits<8>(d, nc, tiles, terms);
            default: return q8_cluster_fits<16>(d, nc, tiles, terms);
        }
    };
    while (splits * terms > 8 && !fits((int)(splits * terms))) splits--;
    Q8GemvArgs p;
    p.slice_len = (chunks + splits - 1) / splits * kQChunk;
    splits = (g.k + p.slice_len - 1) / p.slice_len;
    p.splits = (int)splits;
    p.terms = terms;
    const int nc = p.splits * terms, F = (int)g.m * kQCols;
    p.band = ((F + nc - 1) / nc + 3) / 4 * 4;
    p.out = g.out;
    p.addend = g.addend;
    p.addend_mode = g.addend_mode;
    p.m = g.m;
    p.n = g.n;
    p.k = g.k;
    p.error = d->flags + 2;
    for (int t = 0; t < 2; t++) {
        const Buffer* w = g.packed[t < terms ? t : 0];
        p.quants[t] = static_cast<const int8_t*>(w->ptr);
        p.scales[t] = w->q8_scales;
    }
    p.chunks = chunks;
    CUtensorMap map_a;
    MG_TRY(q8_map(&map_a, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, const_cast<float*>(g.a), g.k, g.m, g.k * 4, kQChunk,
                  (uint32_t)mp, CU_TENSOR_MAP_SWIZZLE_NONE));
    if (tiles > 0x7FFFFFFFull) return fail(MG_SHAPE_UNSUPPORTED, "packed gemv n %llu is too wide", (unsigned long long)g.n);
    dim3 grid((unsigned)tiles, (unsigned)splits, (unsigned)terms);
    switch (mp) {
        case 1: return launch_q8_gemv<1>(d, grid, map_a, p);
        case 2: return launch_q8_gemv<2>(d, grid, map_a, p);
        case 4: return launch_q8_gemv<4>(d, grid, map_a, p);
        case 8: return launch_q8_gemv<8>(d, grid, map_a, p);
        default: return launch_q8_gemv<16>(d, grid, map_a, p);
    }
}

// A matmul with packed B (src/kernels.rs:5581-5600): the few-row kernel when eligible, else each
// packed weight dequantized (stored order) for the duration of the call and the f32 matmul.
bool gemv_tc_q8_eligible(const GemmArgs& g);
mg_status gemv_tc_q8(Device* d, const GemmArgs& g);

mg_status q8_matmul(Device* d, const GemmArgs& g) {
    // The tensor-core form (gemv_tc.cu) widens, scales and splits the quants for the MMAs; the
    // CUDA-core kernel below remains for what it does not take.
    if (gemv_tc_q8_eligible(g)) return gemv_tc_q8(d, g);
    if (q8_gemv_eligible(g)) return q8_gemv(d, g);
    // Few rows: the logical [k, n] matrix, which the f32 few-row matmul reads as it lies (it takes
    // no transposed B); more rows: the stored matrix (a plain row-major pass) with the transpose
    // folded into B's flag for the tensor-core matmul.
    const bool logical = g.m <= 16;
    GemmArgs f = g;
    void* mem[2] = {nullptr, nullptr};
    mg_status s = MG_OK;
    for (int t = 0; t < 2 && s == MG_OK; t++) {
        const Buffer* w = g.packed[t];
        if (!w) continue;
        s = device_alloc(d, w->q8_rows * w->q8_cols * sizeof(float), &mem[t]);
        if (s == MG_OK) s = q8_dequantize(d, w, static_cast<float*>(mem[t]), !logical);
        (t == 0 ? f.b : f.b2) = static_cast<const float*>(mem[t]);
        f.packed[t] = nullptr;
    }
    if (s == MG_OK) {
        // the stored matrix is the logical B, or its transpose for a transposed-storage weight;
        // a gated pair with one packed and one f32 weight is dequantized only when both agree
        const Buffer* w = g.packed[0] ? g.packed[0] : g.packed[1];
        const bool flip = !logical && w->q8_transposed != 0;
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
