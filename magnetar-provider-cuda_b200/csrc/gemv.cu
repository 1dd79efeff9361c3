// matmul for few rows (M <= 16): the decode-side GEMV path, bound by streaming B once.
//
// The reference gives each output column a 16-warp split-K over k with a fixed-order
// combine (src/kernels.cu:1351-1391, 1460-1513: `matmul_split_k{,_rows}_kernel`).  Here a
// CTA owns a 128-column tile of B and one slice of k; each warp streams whole 512-byte rows
// of its tile with 16-byte loads (four rows in flight per warp) and applies them to every
// row of A, which sits in shared memory.  Warps combine in a fixed order, each CTA writes
// one partial per (slice, row, column) to a workspace, and a second kernel sums the slices
// in slice order and applies the addend (bias row / residual) or the SwiGLU gate -- so the
// result is deterministic, and B (the 64 MB weight at K = N = 4096) is read exactly once.
#include <cooperative_groups.h>
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "internal.h"
#include "sm100.cuh"

namespace mg {
namespace {

constexpr int kMaxRows = 16;     // M handled by this path
constexpr int kCols = 128;       // columns per CTA: 32 lanes x float4
constexpr int kWarps = 8;
constexpr int kRowsInFlight = 4; // B rows each warp loads before using them

__device__ __forceinline__ float4 ld_stream(const float4* p) {
    float4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}

// partial[(z * slices + slice) * m * n + row * n + col]; z selects B (0) or B2 (1).
template <int M>
__global__ void __launch_bounds__(kWarps * 32) gemv_partial_kernel(const float* __restrict__ a,
                                                                    const float* __restrict__ b,
                                                                    const float* __restrict__ b2,
                                                                    float* __restrict__ partial, uint64_t m,
                                                                    uint64_t n, uint64_t k, uint64_t slice_len,
                                                                    int transpose_a) {
    pdl_enter();
    extern __shared__ float smem[];
    float* a_s = smem;                      // [M][slice_len]
    float* red = smem + M * slice_len;      // [kWarps][kCols]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint64_t col0 = (uint64_t)blockIdx.x * kCols;
    const uint64_t slice = blockIdx.y;
    const uint64_t k0 = slice * slice_len;
    const uint64_t k1 = min(k, k0 + slice_len);
    const float* w = blockIdx.z ? b2 : b;

    // Stage A[:, k0:k1] (transposed storage reads A^T[k][m]).
    for (uint64_t i = threadIdx.x; i < (uint64_t)M * slice_len; i += blockDim.x) {
        const uint64_t r = i / slice_len, kk = k0 + i % slice_len;
        float v = 0.0f;
        if (r < m && kk < k1) v = transpose_a ? a[kk * m + r] : a[r * k + kk];
        a_s[i] = v;
    }
    __syncthreads();

    const uint64_t col = col0 + 4 * lane;
    const bool full = col + 3 < n;
    float acc[M][4];
#pragma unroll
    for (int r = 0; r < M; r++) acc[r][0] = acc[r][1] = acc[r][2] = acc[r][3] = 0.0f;

    uint64_t kk = k0 + warp;
    for (; kk + (kRowsInFlight - 1) * kWarps < k1; kk += kRowsInFlight * kWarps) {
        float4 bv[kRowsInFlight];
#pragma unroll
        for (int u = 0; u < kRowsInFlight; u++) {
            const float* rowp = w + (kk + u * kWarps) * n + col;
            if (full) bv[u] = ld_stream(reinterpret_cast<const float4*>(rowp));
            else {
                bv[u].x = col < n ? rowp[0] : 0.f;
                bv[u].y = col + 1 < n ? rowp[1] : 0.f;
                bv[u].z = col + 2 < n ? rowp[2] : 0.f;
                bv[u].w = 0.f;
            }
        }
#pragma unroll
        for (int u = 0; u < kRowsInFlight; u++) {
            const uint64_t kl = kk + u * kWarps - k0;
#pragma unroll
            for (int r = 0; r < M; r++) {
                const float av = a_s[r * slice_len + kl];
                acc[r][0] += av * bv[u].x;
                acc[r][1] += av * bv[u].y;
                acc[r][2] += av * bv[u].z;
                acc[r][3] += av * bv[u].w;
            }
        }
    }
    for (; kk < k1; kk += kWarps) {
        const float* rowp = w + kk * n + col;
        float4 bv;
        if (full) bv = ld_stream(reinterpret_cast<const float4*>(rowp));
        else {
            bv.x = col < n ? rowp[0] : 0.f;
            bv.y = col + 1 < n ? rowp[1] : 0.f;
            bv.z = col + 2 < n ? rowp[2] : 0.f;
            bv.w = 0.f;
        }
        const uint64_t kl = kk - k0;
#pragma unroll
        for (int r = 0; r < M; r++) {
            const float av = a_s[r * slice_len + kl];
            acc[r][0] += av * bv.x;
            acc[r][1] += av * bv.y;
            acc[r][2] += av * bv.z;
            acc[r][3] += av * bv.w;
        }
    }

    // Fixed-order combine of the warps, one output row at a time.
    float* out_base = partial + ((uint64_t)blockIdx.z * gridDim.y + slice) * m * n;
#pragma unroll
    for (int r = 0; r < M; r++) {
        if (r >= (int)m) break;
        __syncthreads();
        *reinterpret_cast<float4*>(&red[warp * kCols + 4 * lane]) =
            make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
        __syncthreads();
        if (threadIdx.x < kCols) {
            float s = 0.0f;
#pragma unroll
            for (int wi = 0; wi < kWarps; wi++) s += red[wi * kCols + threadIdx.x];
            const uint64_t c = col0 + threadIdx.x;
            if (c < n) out_base[r * n + c] = s;
        }
    }
}

// out = sum over slices (in order) [+ addend] or silu(gate) * up when gated.
__global__ void __launch_bounds__(256) gemv_reduce_kernel(const float* __restrict__ partial, float* __restrict__ out,
                                                          uint64_t m, uint64_t n, uint64_t slices,
                                                          const float* __restrict__ addend, int addend_mode,
                                                          int gated) {
    pdl_enter();
    const uint64_t total = m * n;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
        float s = 0.0f;
        for (uint64_t sl = 0; sl < slices; sl++) s += partial[sl * total + i];
        if (gated) {
            float u = 0.0f;
            for (uint64_t sl = 0; sl < slices; sl++) u += partial[(slices + sl) * total + i];
            s = (s * (1.0f / (1.0f + expf(-s)))) * u;
        } else if (addend_mode == 1) {
            s += addend[i % n];
        } else if (addend_mode == 2) {
            s += addend[i];
        }
        out[i] = s;
    }
}

template <int M>
void launch_partial(Device* d, dim3 grid, size_t smem, const k::GemmArgs& g, float* partial, uint64_t slice_len) {
    enqueue(d, gemv_partial_kernel<M>, grid, kWarps * 32, smem, g.a, g.b, g.b2, partial, g.m, g.n, g.k, slice_len,
                                                                   g.transpose_a);
}

// ---- TMA-staged streaming of B ---------------------------------------------------------------
// A producer lane streams [kChunkRows x 128] tiles of B (16 KB) into a kStages-deep shared
// ring with TMA; every warp takes 4 consecutive rows of each tile and multiplies them by the
// matching 4 columns of A (one 16-byte shared load per row of A), so ~96 KB of B is in flight
// per CTA regardless of the warps' arithmetic.
constexpr int kChunkRows = 32;
constexpr int kStages = 4;      // 64 KB of B in flight per CTA; two CTAs fit an SM
constexpr int kMaxSlices = 32;  // k slices per column tile (the last CTA's sum loads them at once)
constexpr int kChunkBytes = kChunkRows * kCols * 4;
constexpr uint64_t kMaxCounterTiles = 1u << 16;  // Device::counters entries

struct GemvTmaArgs {
    const float* a;
    float* partial;  // [zs][slices][m][n]
    float* out;
    const float* addend;
    int addend_mode;
    int gated;
    uint64_t m, n, k, slice_len;
    int transpose_a;
    int* error;
    unsigned int* counters;  // per column tile; zero between calls (the last CTA resets it)
};

// Warps 0-7 compute; warp 8 is the TMA producer.  The last CTA to finish a column tile sums
// that tile's partials over the slices (in slice order) and writes the output, so no second
// kernel is needed.
template <int M>
__global__ void __launch_bounds__((kWarps + 1) * 32, 2) gemv_tma_kernel(const __grid_constant__ CUtensorMap map_b,
                                                                      const __grid_constant__ CUtensorMap map_b2,
                                                                      GemvTmaArgs p) {
    pdl_enter();
    extern __shared__ uint8_t smem_raw[];
    using namespace sm100;
    __shared__ unsigned int s_last;
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 127u) & ~127u;
    uint8_t* base_ptr = smem_raw + (base - raw);
    float* ring = reinterpret_cast<float*>(base_ptr);                        // [kStages][32][128]
    float* a_s = ring + kStages * kChunkRows * kCols;                          // [M][slice_len]
    float* red = a_s + M * p.slice_len;                                        // [kWarps][kCols]
    uint64_t* bars = reinterpret_cast<uint64_t*>(red + kWarps * kCols);        // full[kStages], empty[kStages]
    const uint32_t bar0 = smem_u32(bars);
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (kStages + s); };
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint64_t m = p.m, n = p.n, k = p.k, slice_len = p.slice_len;
    const uint64_t col0 = (uint64_t)blockIdx.x * kCols;
    const uint64_t slice = blockIdx.y;
    const uint64_t k0 = slice * slice_len;
    const uint64_t k1 = min(k, k0 + slice_len);
    const int chunks = (int)((k1 - k0 + kChunkRows - 1) / kChunkRows);
    const CUtensorMap* map = blockIdx.z ? &map_b2 : &map_b;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), kWarps);
        }
        fence_barrier_init();
    }
    // Stage A[:, k0:k1] (zero past k1 so a partial last tile multiplies zero rows of B), with
    // several loads in flight per thread: 16-byte loads when A's rows allow them.
    if (!p.transpose_a && k % 4 == 0 && k0 % 4 == 0 && (reinterpret_cast<uintptr_t>(p.a) & 15) == 0) {
        const uint64_t q = slice_len / 4;  // float4 per staged row (slice_len is a multiple of 32)
        const uint64_t total = (uint64_t)M * q;
        for (uint64_t i0 = threadIdx.x; i0 < total; i0 += 4 * blockDim.x) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const uint64_t i = i0 + (uint64_t)u * blockDim.x;
                const uint64_t r = i / q, kk = k0 + 4 * (i % q);
                v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (i < total && r < m && kk < k1) v[u] = *reinterpret_cast<const float4*>(p.a + r * k + kk);
            }
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const uint64_t i = i0 + (uint64_t)u * blockDim.x;
                if (i < total) reinterpret_cast<float4*>(a_s)[i] = v[u];
            }
        }
    } else {
        for (uint64_t i0 = threadIdx.x; i0 < (uint64_t)M * slice_len; i0 += 4 * blockDim.x) {
            float v[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const uint64_t i = i0 + (uint64_t)u * blockDim.x;
                const uint64_t r = i / slice_len, kk = k0 + i % slice_len;
                v[u] = 0.0f;
                if (i < (uint64_t)M * slice_len && r < m && kk < k1) v[u] = p.transpose_a ? p.a[kk * m + r] : p.a[r * k + kk];
            }
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const uint64_t i = i0 + (uint64_t)u * blockDim.x;
                if (i < (uint64_t)M * slice_len) a_s[i] = v[u];
            }
        }
    }
    __syncthreads();

    float acc[M][4];
#pragma unroll
    for (int r = 0; r < M; r++) acc[r][0] = acc[r][1] = acc[r][2] = acc[r][3] = 0.0f;
    if (warp == kWarps) {
        // ---- producer: keep the ring full -------------------------------------------------
        if (lane == 0) {
            prefetch_tensormap(map);
            for (int c = 0; c < chunks; c++) {
                const int s = c % kStages;
                if (c >= kStages && !mbar_wait(empty_bar(s), (uint32_t)(c / kStages - 1) & 1u)) {
                    atomicExch(p.error, 1);
                    break;
                }
                mbar_arrive_expect_tx(full_bar(s), kChunkBytes);
                tma_load_2d(base + (uint32_t)(s * kChunkBytes), map, full_bar(s), (int)col0,
                            (int)(k0 + (uint64_t)c * kChunkRows));
            }
        }
        __syncwarp();
    } else {
        for (int c = 0; c < chunks; c++) {
            const int s = c % kStages;
            const uint32_t phase = (uint32_t)(c / kStages) & 1u;
            if (!mbar_wait(full_bar(s), phase)) {
                atomicExch(p.error, 1);
                break;
            }
            const float* tile = ring + s * kChunkRows * kCols;
            const int rr = warp * 4;  // this warp's 4 rows of the tile
            float4 bv[4];
#pragma unroll
            for (int u = 0; u < 4; u++) bv[u] = *reinterpret_cast<const float4*>(tile + (rr + u) * kCols + 4 * lane);
            __syncwarp();
            if (lane == 0) mbar_arrive(empty_bar(s));  // the stage's data is in registers
            const uint64_t kl = (uint64_t)c * kChunkRows + rr;  // row within the slice (multiple of 4)
#pragma unroll
            for (int r = 0; r < M; r++) {
                const float4 av = *reinterpret_cast<const float4*>(a_s + r * slice_len + kl);
                const float aa[4] = {av.x, av.y, av.z, av.w};
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    acc[r][0] += aa[u] * bv[u].x;
                    acc[r][1] += aa[u] * bv[u].y;
                    acc[r][2] += aa[u] * bv[u].z;
                    acc[r][3] += aa[u] * bv[u].w;
                }
            }
        }
    }
    // Fixed-order combine of the warps, one output row at a time.
    float* out_base = p.partial + ((uint64_t)blockIdx.z * gridDim.y + slice) * m * n;
#pragma unroll
    for (int r = 0; r < M; r++) {
        if (r >= (int)m) break;
        __syncthreads();
        if (warp < kWarps)
            *reinterpret_cast<float4*>(&red[warp * kCols + 4 * lane]) =
                make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
        __syncthreads();
        if (threadIdx.x < kCols) {
            float sum = 0.0f;
#pragma unroll
            for (int wi = 0; wi < kWarps; wi++) sum += red[wi * kCols + threadIdx.x];
            const uint64_t cidx = col0 + threadIdx.x;
            if (cidx < n) out_base[r * n + cidx] = sum;
        }
    }
    // The last CTA of this column tile (over slices and gate/up) finishes it.
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned int total = gridDim.y * gridDim.z;
        s_last = atomicAdd(&p.counters[blockIdx.x], 1u) == total - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const int slices = (int)gridDim.y;  // <= kMaxSlices
    const uint64_t mn = m * n;
    // Sum over the slices in slice order, eight slices' partials loaded before they are added
    // (eight loads in flight at once).
    auto sum_slices = [&](int zs, uint64_t off) {
        float acc = 0.0f;
        for (int sl0 = 0; sl0 < slices; sl0 += 8) {
            float t[8];
#pragma unroll
            for (int u = 0; u < 8; u++)
                if (sl0 + u < slices) t[u] = __ldcg(p.partial + ((uint64_t)zs * slices + sl0 + u) * mn + off);
#pragma unroll
            for (int u = 0; u < 8; u++)
                if (sl0 + u < slices) acc += t[u];
        }
        return acc;
    };
    for (uint64_t i = threadIdx.x; i < m * kCols; i += blockDim.x) {
        const uint64_t r = i / kCols, cidx = col0 + i % kCols;
        if (cidx >= n) continue;
        const uint64_t off = r * n + cidx;
        float s = sum_slices(0, off);
        if (p.gated) {
            const float u = sum_slices(1, off);
            s = (s * (1.0f / (1.0f + expf(-s)))) * u;
        } else if (p.addend_mode == 1) {
            s += p.addend[cidx];
        } else if (p.addend_mode == 2) {
            s += p.addend[off];
        }
        p.out[off] = s;
    }
    if (threadIdx.x == 0) p.counters[blockIdx.x] = 0u;
}

PFN_cuTensorMapEncodeTiled_v12000 gemv_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// Row-major [k, n] f32 B, box [kChunkRows x kCols], no swizzle.
mg_status gemv_map(CUtensorMap* map, const float* b, uint64_t k, uint64_t n) {
    auto fn = gemv_encode_fn();
    if (!fn) return mg::fail(MG_DRIVER_FAILED, "the driver does not provide cuTensorMapEncodeTiled");
    cuuint64_t dims[2] = {n, k};
    cuuint64_t strides[1] = {n * sizeof(float)};
    cuuint32_t box[2] = {kCols, kChunkRows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(b), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return mg::fail(MG_DRIVER_FAILED, "encoding a TMA descriptor failed (CUresult %d)", (int)r);
    return MG_OK;
}

// ---- cluster GEMV: A and B streamed together, k split across a thread-block cluster -----------
// A producer lane streams, per stage, a [32 x 128] tile of B and the matching [M x 32] columns
// of A with TMA (no prologue staging A); 8 compute warps take 4 rows of B each per stage and
// multiply them by A from shared memory, two columns per packed FMA.  When B is a settled
// weight, the first stages' B loads are issued before the dependency wait, so a chain of
// GEMVs streams the next weight while the previous call finishes.  The k slices of one column tile (and, gated, the
// gate and up terms) form one cluster: each CTA sums its warps once through the drained ring,
// then sends each band of its [M x 128] partial to the CTA that owns the band with one bulk
// copy into that CTA's receive slot; owners add the partials in split order (deterministic),
// apply bias / residual / SwiGLU and write.  B is read exactly once; nothing goes through
// global memory but the operands and the result.
constexpr int kCStages = 4;
constexpr int kMaxClusterCtas = 16;  // non-portable cluster size (checked against the GPU at launch)

struct GemvClusterArgs {
    float* out;
    const float* addend;
    int addend_mode;
    uint64_t m, n, k;
    uint64_t slice_len;  // k rows per split (multiple of kChunkRows)
    int splits;          // S; the cluster is (1, S, terms)
    int terms;           // 1, or 2 for gated (gate: z = 0, up: z = 1)
    int band;            // floats of the flattened [m][128] tile each cluster CTA finishes (multiple of 4)
    int b_early;         // B does not depend on the preceding kernel: the first stages' B loads
                         // are issued before the dependency wait
    int* error;
};

// Two f32 lanes at once (Blackwell's packed FMA): d.lo += a * b.lo, d.hi += a * b.hi, each
// lane one fused multiply-add with round-to-nearest, as the scalar form.
__device__ __forceinline__ uint64_t pack2(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void fma2(uint64_t& d, float a, uint64_t b) {
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(d) : "l"(pack2(a, a)), "l"(b));
}
__device__ __forceinline__ void fma2(uint64_t& d, uint64_t a, uint64_t b) {
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(d) : "l"(a), "l"(b));
}
__device__ __forceinline__ float4 unpack4(uint64_t lo, uint64_t hi) {
    float4 v;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(v.x), "=f"(v.y) : "l"(lo));
    asm("mov.b64 {%0, %1}, %2;" : "=f"(v.z), "=f"(v.w) : "l"(hi));
    return v;
}

// From 8 rows up, a transposer warp rewrites each stage's A tile as [32 k][M] so that the
// compute warps read A in pairs of rows (one packed FMA per pair and column, B duplicated
// once per column) instead of duplicating every A value.
//
// H: B is a compact weight, its values stored as bfloat16 bits (each exactly its f32 value);
// a stage carries half the bytes of B, the ring holds more stages, and each value is widened
// back to the same f32 in registers -- the arithmetic and its order are those of the f32 form,
// so the results are bit-identical.
template <int M, bool H = false>
struct GemvCShape {
    static constexpr bool kTrans = M >= 8;
    // Compute warps: eight along k (four k rows of a stage each) times kMW along the rows of A --
    // at 16 rows two warps share each k slice, eight rows each, so twice the warps hide the latency
    // of the loads and packed FMAs with half the accumulators per thread.
    static constexpr int kMW = M >= 16 && !H ? 2 : 1;  // (the compact form measured slower with 2)
    static constexpr int kCW = kWarps * kMW;
    static constexpr int kQH = M / 4 / kMW;  // groups of four A rows per warp (row-pair form)
    static_assert(kWarps * 4 == kChunkRows, "eight warps of four k rows cover a stage");
    static constexpr int kThreads = (kCW + 1 + (kTrans ? 1 : 0)) * 32;
    // 16 rows hold 64 accumulator registers per thread: one CTA per SM (no spills) with a ring
    // twice as deep; fewer rows, two CTAs per SM.
    static constexpr int kMinBlocks = M >= 16 ? 1 : 2;
    static constexpr int kStages = M >= 16 ? (H ? 14 : 8) : (H ? 8 : kCStages);
    static constexpr int kB = kChunkRows * kCols * (H ? 2 : 4);  // 16 KB (8 KB compact) of B per stage
    static constexpr int kA = M * kChunkRows * 4;      // [M][32] of A per stage
    static constexpr int kStage = kB + kA;
    static constexpr int kRing = kStages * kStage;
    static constexpr int kAT = kTrans ? kStages * kA : 0;  // the transposed A tiles, [32][M] per stage
    static constexpr int kPart = M * kCols * 4;         // this CTA's partial [M][128]
    static constexpr int kRecv = (M * kCols + 4 * kMaxClusterCtas) * 4;  // the other CTAs' partials of this CTA's band
    static_assert(kWarps * kPart <= kRing, "the warp partials fit the drained ring");
    static constexpr int kSmem = 128 + kRing + kAT + kPart + kRecv + 8 * (3 * kStages + 1);
};

// Four consecutive columns of row `row` of a B stage, as f32.
template <bool H>
__device__ __forceinline__ float4 gemv_b4(const uint8_t* tile, int row, int lane) {
    if constexpr (H) {
        const uint2 u = *reinterpret_cast<const uint2*>(tile + (row * kCols + 4 * lane) * 2);
        return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u), __uint_as_float(u.y << 16),
                           __uint_as_float(u.y & 0xFFFF0000u));
    } else {
        return *reinterpret_cast<const float4*>(tile + (row * kCols + 4 * lane) * 4);
    }
}

template <int M, bool H>
__global__ void __launch_bounds__(GemvCShape<M, H>::kThreads, GemvCShape<M, H>::kMinBlocks) gemv_cluster_kernel(const __grid_constant__ CUtensorMap map_a,
                                                                          const __grid_constant__ CUtensorMap map_b,
                                                                          const __grid_constant__ CUtensorMap map_b2,
                                                                          GemvClusterArgs p) {
    using namespace sm100;
    using S = GemvCShape<M, H>;
    constexpr int kCStages = S::kStages;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 127u) & ~127u;
    uint8_t* base_ptr = smem_raw + (base - raw);
    const uint32_t part = base + S::kRing + S::kAT;
    const uint32_t recv = part + S::kPart;
    const uint32_t bar0 = recv + S::kRecv;
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (kCStages + s); };
    const uint32_t recv_bar = bar0 + 8u * (2 * kCStages);
    auto at_bar = [&](int s) { return bar0 + 8u * (2 * kCStages + 1 + s); };  // transposed A ready
    float* atf = reinterpret_cast<float*>(base_ptr + S::kRing);  // [kCStages][32][M]
    float* partf = reinterpret_cast<float*>(base_ptr + S::kRing + S::kAT);
    float* recvf = reinterpret_cast<float*>(base_ptr + S::kRing + S::kAT + S::kPart);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint64_t col0 = (uint64_t)blockIdx.x * kCols;
    const int nc = p.splits * p.terms;
    const int rank = (int)cooperative_groups::this_cluster().block_rank();
    const uint64_t k0 = (uint64_t)blockIdx.y * p.slice_len;
    const uint64_t k1 = min(p.k, k0 + p.slice_len);
    const int chunks = k1 > k0 ? (int)((k1 - k0 + kChunkRows - 1) / kChunkRows) : 0;
    const int F = (int)p.m * kCols;
    const int my_lo = min(F, rank * p.band), my_hi = min(F, my_lo + p.band);
    const CUtensorMap* mb = blockIdx.z ? &map_b2 : &map_b;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kCStages; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), S::kCW);
            if (S::kTrans) mbar_init(at_bar(s), 1);
        }
        mbar_init(recv_bar, 1);
        fence_barrier_init();
        mbar_arrive_expect_tx(recv_bar, (uint32_t)((nc - 1) * (my_hi - my_lo) * 4));
        if (p.b_early) {
            for (int c = 0; c < min(chunks, kCStages); c++) {
                mbar_arrive_expect_tx(full_bar(c), (uint32_t)S::kStage);
                tma_load_2d(base + (uint32_t)(c * S::kStage), mb, full_bar(c), (int)col0, (int)(k0 + (uint64_t)c * kChunkRows));
            }
        }
    }
    cluster_arrive();  // phase 1: every CTA's receive barrier is armed before anyone sends
    pdl_enter();
    __syncthreads();

    // Packed f32 accumulators of this thread's 4 columns: [row][column pair] below 8 rows,
    // [row pair][column] from 8 rows up.
    constexpr int kAcc = S::kTrans ? 8 * S::kQH : 2 * M;
    uint64_t acc2[kAcc];
#pragma unroll
    for (int i = 0; i < kAcc; i++) acc2[i] = 0ull;
    if (S::kTrans && warp == S::kCW + 1) {
        // ---- transposer: A [M][32] -> [32][M] per stage (lane = k) ---------------------------
        for (int c = 0; c < chunks; c++) {
            const int s = c % kCStages;
            if (!mbar_wait(full_bar(s), (uint32_t)(c / kCStages) & 1u)) {
                atomicExch(p.error, 1);
                break;
            }
            const float* at = reinterpret_cast<const float*>(base_ptr + s * S::kStage + S::kB);
            float* dst = atf + (s * kChunkRows + lane) * M;
#pragma unroll
            for (int q = 0; q < M / 4; q++)
                *reinterpret_cast<float4*>(dst + 4 * q) = make_float4(at[(4 * q) * kChunkRows + lane], at[(4 * q + 1) * kChunkRows + lane],
                                                                      at[(4 * q + 2) * kChunkRows + lane], at[(4 * q + 3) * kChunkRows + lane]);
            __syncwarp();
            if (lane == 0) mbar_arrive(at_bar(s));
        }
    } else if (warp == S::kCW) {
        // ---- producer: keep the ring full -----------------------------------------------
        if (lane == 0) {
            for (int c = 0; c < chunks; c++) {
                const int s = c % kCStages;
                if (c >= kCStages && !mbar_wait(empty_bar(s), (uint32_t)(c / kCStages - 1) & 1u)) {
                    atomicExch(p.error, 1);
                    break;
                }
                const uint32_t st = base + (uint32_t)(s * S::kStage);
                const int kr = (int)(k0 + (uint64_t)c * kChunkRows);
                if (!p.b_early || c >= kCStages) {
                    mbar_arrive_expect_tx(full_bar(s), (uint32_t)S::kStage);
                    tma_load_2d(st, mb, full_bar(s), (int)col0, kr);
                }
                tma_load_2d(st + S::kB, &map_a, full_bar(s), kr, 0);
            }
        }
        __syncwarp();
    } else if (warp < S::kCW) {
        for (int c = 0; c < chunks; c++) {
            const int s = c % kCStages;
            const uint32_t ph = (uint32_t)(c / kCStages) & 1u;
            if (!mbar_wait(full_bar(s), ph) || (S::kTrans && !mbar_wait(at_bar(s), ph))) {
                atomicExch(p.error, 1);
                break;
            }
            const uint8_t* tile = base_ptr + s * S::kStage;
            const int rr = (warp % kWarps) * 4;  // this warp's k rows of the stage
            const int rh = warp / kWarps;         // and its share of A's rows
            if constexpr (S::kTrans) {
                const float* att = atf + s * kChunkRows * M;  // [32][M]
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const float4 bv = gemv_b4<H>(tile, rr + u, lane);
                    const uint64_t bd[4] = {pack2(bv.x, bv.x), pack2(bv.y, bv.y), pack2(bv.z, bv.z), pack2(bv.w, bv.w)};
#pragma unroll
                    for (int q = 0; q < S::kQH; q++) {
                        const float4 a4 = *reinterpret_cast<const float4*>(att + (rr + u) * M + 4 * (rh * S::kQH + q));
                        const uint64_t a01 = pack2(a4.x, a4.y), a23 = pack2(a4.z, a4.w);
#pragma unroll
                        for (int cc = 0; cc < 4; cc++) {
                            fma2(acc2[(2 * q) * 4 + cc], a01, bd[cc]);
                            fma2(acc2[(2 * q + 1) * 4 + cc], a23, bd[cc]);
                        }
                    }
                }
            } else {
                const float* at = reinterpret_cast<const float*>(base_ptr + s * S::kStage + S::kB);  // [M][32]
                uint64_t b01[4], b23[4];
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const float4 bv = gemv_b4<H>(tile, rr + u, lane);
                    b01[u] = pack2(bv.x, bv.y);
                    b23[u] = pack2(bv.z, bv.w);
                }
#pragma unroll
                for (int r = 0; r < M; r++) {
                    const float4 av = *reinterpret_cast<const float4*>(at + r * kChunkRows + rr);
                    const float aa[4] = {av.x, av.y, av.z, av.w};
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        fma2(acc2[r * 2], aa[u], b01[u]);
                        fma2(acc2[r * 2 + 1], aa[u], b23[u]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty_bar(s));  // this warp is done with the stage
        }
    }
    // ---- this CTA's partial: the warps' sums in warp order, through the drained ring ----------
    __syncthreads();
    float* red = reinterpret_cast<float*>(base_ptr);  // [k warps][M][128]
    if (warp < S::kCW) {
        if constexpr (S::kTrans) {
            // acc2[q * 4 + cc] holds rows 2q, 2q + 1 of this warp's share, column cc
            const int kw = warp % kWarps, r0 = (warp / kWarps) * 4 * S::kQH;
#pragma unroll
            for (int q = 0; q < 2 * S::kQH; q++) {
                float lo[4], hi[4];
#pragma unroll
                for (int cc = 0; cc < 4; cc++)
                    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo[cc]), "=f"(hi[cc]) : "l"(acc2[q * 4 + cc]));
                *reinterpret_cast<float4*>(red + (kw * M + r0 + 2 * q) * kCols + 4 * lane) = make_float4(lo[0], lo[1], lo[2], lo[3]);
                *reinterpret_cast<float4*>(red + (kw * M + r0 + 2 * q + 1) * kCols + 4 * lane) = make_float4(hi[0], hi[1], hi[2], hi[3]);
            }
        } else {
#pragma unroll
            for (int r = 0; r < M; r++)
                *reinterpret_cast<float4*>(red + (warp * M + r) * kCols + 4 * lane) = unpack4(acc2[r * 2], acc2[r * 2 + 1]);
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < F; i += blockDim.x) {
        const int r = i / kCols, c = i % kCols;
        float sum = 0.0f;
#pragma unroll
        for (int w = 0; w < kWarps; w++) sum += red[(w * M + r) * kCols + c];
        partf[i] = sum;
    }
    fence_proxy_async();  // the partial is read by bulk copies next
    __syncthreads();
    // ---- exchange: each band of the partial to the CTA that owns it ---------------------------
    cluster_wait();  // phase 1
    if (threadIdx.x == 0) {
        for (int o = 0; o < nc; o++) {
            if (o == rank) continue;
            const int lo = min(F, o * p.band), hi = min(F, lo + p.band);
            if (hi > lo)
                bulk_copy_to_cluster(mapa(recv + (uint32_t)(rank * p.band * 4), (uint32_t)o), part + (uint32_t)(lo * 4),
                                     (uint32_t)((hi - lo) * 4), mapa(recv_bar, (uint32_t)o));
        }
    }
    if (!mbar_wait(recv_bar, 0)) atomicExch(p.error, 1);
    cluster_arrive();  // phase 2: every copy into this CTA has landed
    // ---- finish this CTA's band: splits in order, per term -----------------------------------
    for (int e = my_lo + (int)threadIdx.x; e < my_hi; e += blockDim.x) {
        const int r = e / kCols, c = e % kCols;
        const uint64_t col = col0 + c;
        if (col >= p.n) continue;
        auto from = [&](int src) { return src == rank ? partf[e] : recvf[src * p.band + (e - my_lo)]; };
        float g = 0.0f;
        for (int s = 0; s < p.splits; s++) g += from(s);
        float v;
        if (p.terms == 2) {
            float u = 0.0f;
            for (int s = 0; s < p.splits; s++) u += from(p.splits + s);
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

// Row-major [k, n] bfloat16 bits of a compact B, box [kChunkRows x kCols], no swizzle.
mg_status gemv_map_compact(CUtensorMap* map, const uint16_t* b, uint64_t k, uint64_t n) {
    auto fn = gemv_encode_fn();
    if (!fn) return mg::fail(MG_DRIVER_FAILED, "the driver does not provide cuTensorMapEncodeTiled");
    cuuint64_t dims[2] = {n, k};
    cuuint64_t strides[1] = {n * sizeof(uint16_t)};
    cuuint32_t box[2] = {kCols, kChunkRows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint16_t*>(b), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return mg::fail(MG_DRIVER_FAILED, "encoding a TMA descriptor failed (CUresult %d)", (int)r);
    return MG_OK;
}

// Row-major [m, k] f32 A, box [32 x mp] (rows past m read as zero).
mg_status gemv_a_map(CUtensorMap* map, const float* a, uint64_t m, uint64_t k, uint32_t mp) {
    auto fn = gemv_encode_fn();
    if (!fn) return mg::fail(MG_DRIVER_FAILED, "the driver does not provide cuTensorMapEncodeTiled");
    cuuint64_t dims[2] = {k, m};
    cuuint64_t strides[1] = {k * sizeof(float)};
    cuuint32_t box[2] = {kChunkRows, mp};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(a), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return mg::fail(MG_DRIVER_FAILED, "encoding a TMA descriptor failed (CUresult %d)", (int)r);
    return MG_OK;
}

// k slices of `splits` CTAs each, and the band of the output tile each cluster CTA finishes.
void gemv_slices(GemvClusterArgs& p, uint64_t splits) {
    const uint64_t kb = (p.k + kChunkRows - 1) / kChunkRows;
    if (splits > kb) splits = kb;
    if (splits < 1) splits = 1;
    p.slice_len = ((kb + splits - 1) / splits) * kChunkRows;
    p.splits = (int)((p.k + p.slice_len - 1) / p.slice_len);
    if (p.splits < 1) p.splits = 1;
    const int nc = p.splits * p.terms, F = (int)p.m * kCols;
    p.band = ((F + nc - 1) / nc + 3) / 4 * 4;
}

template <int M, bool H>
mg_status launch_cluster(Device* d, GemvClusterArgs p, uint64_t col_tiles, const CUtensorMap* maps) {
    using S = GemvCShape<M, H>;
    static bool configured[64] = {false};
    if (!configured[d->ordinal & 63]) {
        MG_CUDA(cudaFuncSetAttribute(gemv_cluster_kernel<M, H>, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmem),
                "configuring the cluster gemv kernel");
        MG_CUDA(cudaFuncSetAttribute(gemv_cluster_kernel<M, H>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1),
                "allowing the cluster gemv kernel clusters of up to 16");
        configured[d->ordinal & 63] = true;
    }
    // Clusters larger than 8 only where the GPU holds them all in one wave (queried once per
    // size); otherwise fewer k splits.
    static int fits[kMaxClusterCtas + 1] = {0};  // 1 fits, -1 does not
    while (p.splits * p.terms > 8) {
        const int nc = p.splits * p.terms;
        if (fits[nc] == 0) {
            cudaLaunchConfig_t q = {};
            q.gridDim = dim3((unsigned)col_tiles, (unsigned)p.splits, (unsigned)p.terms);
            q.blockDim = dim3(S::kThreads, 1, 1);
            q.dynamicSmemBytes = S::kSmem;
            cudaLaunchAttribute ca;
            ca.id = cudaLaunchAttributeClusterDimension;
            ca.val.clusterDim.x = 1;
            ca.val.clusterDim.y = (unsigned)p.splits;
            ca.val.clusterDim.z = (unsigned)p.terms;
            q.attrs = &ca;
            q.numAttrs = 1;
            int clusters = 0;
            if (cudaOccupancyMaxActiveClusters(&clusters, gemv_cluster_kernel<M, H>, &q) != cudaSuccess) {
                (void)cudaGetLastError();
                clusters = 0;
            }
            fits[nc] = (uint64_t)clusters >= col_tiles ? 1 : -1;
        }
        if (fits[nc] > 0) break;
        gemv_slices(p, (uint64_t)p.splits - 1);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)col_tiles, (unsigned)p.splits, (unsigned)p.terms);
    cfg.blockDim = dim3(S::kThreads, 1, 1);
    cfg.dynamicSmemBytes = S::kSmem;
    cfg.stream = d->stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = (unsigned)p.splits;
    attr[0].val.clusterDim.z = (unsigned)p.terms;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = d->pdl ? 2 : 1;
    MG_CUDA(cudaLaunchKernelEx(&cfg, gemv_cluster_kernel<M, H>, maps[0], maps[1], maps[2], p), "cluster gemv launch");
    return launched(d, "cluster gemv launch");
}

// dst[i] = the bfloat16 bits of src[i]; *not_exact is set when some value is not exactly a
// bfloat16 value (nonzero low 16 bits), and dst is then not used.
__global__ void __launch_bounds__(256) compact_bf16_kernel(const float4* __restrict__ src, uint2* __restrict__ dst,
                                                           uint64_t quads, int* not_exact) {
    pdl_enter();  // the weight may have just been written by the kernel before this one
    uint32_t low = 0;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < quads; i += (uint64_t)gridDim.x * blockDim.x) {
        const float4 v = src[i];
        const uint32_t x = __float_as_uint(v.x), y = __float_as_uint(v.y), z = __float_as_uint(v.z), w = __float_as_uint(v.w);
        low |= (x | y | z | w) & 0xFFFFu;
        dst[i] = make_uint2((x >> 16) | (y & 0xFFFF0000u), (z >> 16) | (w & 0xFFFF0000u));
    }
    if (__syncthreads_or(low != 0) && threadIdx.x == 0) atomicExch(not_exact, 1);
}

}  // namespace

namespace k {

mg_status gemv_compact_b(Device* d, const float* b, uint16_t* dst, uint64_t count, int* not_exact) {
    if (count % 4 != 0 || (reinterpret_cast<uintptr_t>(b) & 15) != 0)
        return fail(MG_LAYOUT_UNSUPPORTED, "a compact weight needs a multiple of 4 values, 16-byte aligned");
    const uint64_t quads = count / 4;
    uint64_t blocks = (quads + 255) / 256;
    if (blocks > (uint64_t)d->sm_count * 8) blocks = (uint64_t)d->sm_count * 8;
    enqueue(d, compact_bf16_kernel, (unsigned)(blocks ? blocks : 1), 256, 0, reinterpret_cast<const float4*>(b),
            reinterpret_cast<uint2*>(dst), quads, not_exact);
    return launched(d, "weight compaction launch");
}

// Eligible when M <= 16, B is not transposed and its rows are 16-byte aligned.
bool gemv_eligible(const GemmArgs& g) {
    return g.m >= 1 && g.m <= kMaxRows && !g.transpose_b && g.n % 4 == 0 &&
           (reinterpret_cast<uintptr_t>(g.b) & 15) == 0 && (!g.b2 || (reinterpret_cast<uintptr_t>(g.b2) & 15) == 0);
}

template <int M>
mg_status launch_tma(Device* d, dim3 grid, size_t smem, const CUtensorMap* maps, const GemmArgs& g, float* partial,
                     uint64_t slice_len) {
    static bool configured[64] = {false};
    if (!configured[d->ordinal & 63]) {
        MG_CUDA(cudaFuncSetAttribute(gemv_tma_kernel<M>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024),
                "configuring the gemv kernel");
        configured[d->ordinal & 63] = true;
    }
    GemvTmaArgs p;
    p.a = g.a;
    p.partial = partial;
    p.out = g.out;
    p.addend = g.addend;
    p.addend_mode = g.addend_mode;
    p.gated = g.gated;
    p.m = g.m;
    p.n = g.n;
    p.k = g.k;
    p.slice_len = slice_len;
    p.transpose_a = g.transpose_a;
    p.error = d->flags + 2;
    p.counters = d->counters;
    enqueue(d, gemv_tma_kernel<M>, grid, (kWarps + 1) * 32, smem, maps[0], maps[1], p);
    return launched(d, "gemv kernel launch");
}

// The TMA-staged path: one wave of CTAs (two per SM), each streaming one k-slice of one
// 128-column tile of B; eligible when the k slices needed for that fit kMaxSlices with A's
// slice in shared memory.
bool gemv_tma_plan(const Device* d, const GemmArgs& g, uint64_t* slices_out, uint64_t* slice_len_out) {
    const uint64_t col_tiles = (g.n + kCols - 1) / kCols;
    const int zs = g.gated ? 2 : 1;
    const int mp = g.m <= 1 ? 1 : g.m <= 2 ? 2 : g.m <= 4 ? 4 : g.m <= 8 ? 8 : 16;
    const uint64_t max_slice = (uint64_t)(8192 / mp) / kChunkRows * kChunkRows;  // A's slice <= 32 KB
    if (col_tiles > kMaxCounterTiles) return false;
    uint64_t slices = (uint64_t)d->sm_count * 2 / zs / col_tiles;
    if (slices < 1) slices = 1;
    if (slices > (uint64_t)kMaxSlices) slices = kMaxSlices;
    uint64_t slice_len = (g.k + slices - 1) / slices;
    slice_len = ((slice_len + kChunkRows - 1) / kChunkRows) * kChunkRows;
    if (slice_len > max_slice) slice_len = max_slice;
    slices = (g.k + slice_len - 1) / slice_len;
    if (slices > (uint64_t)kMaxSlices) return false;
    *slices_out = slices;
    *slice_len_out = slice_len;
    return true;
}

mg_status gemv_tma(Device* d, const GemmArgs& g, uint64_t slices, uint64_t slice_len) {
    const uint64_t col_tiles = (g.n + kCols - 1) / kCols;
    const int zs = g.gated ? 2 : 1;
    const int mp = g.m <= 1 ? 1 : g.m <= 2 ? 2 : g.m <= 4 ? 4 : g.m <= 8 ? 8 : 16;
    const size_t smem = 128 + (size_t)kStages * kChunkBytes + ((size_t)mp * slice_len + kWarps * kCols) * sizeof(float) +
                        2 * kStages * sizeof(uint64_t);
    float* partial = nullptr;
    MG_TRY(scratch(d, 0, (size_t)zs * slices * g.m * g.n * sizeof(float), (void**)&partial));
    CUtensorMap maps[2];
    MG_TRY(gemv_map(&maps[0], g.b, g.k, g.n));
    if (g.gated) MG_TRY(gemv_map(&maps[1], g.b2, g.k, g.n));
    else maps[1] = maps[0];
    dim3 grid((unsigned)col_tiles, (unsigned)slices, (unsigned)zs);
    switch (mp) {
        case 1: MG_TRY(launch_tma<1>(d, grid, smem, maps, g, partial, slice_len)); break;
        case 2: MG_TRY(launch_tma<2>(d, grid, smem, maps, g, partial, slice_len)); break;
        case 4: MG_TRY(launch_tma<4>(d, grid, smem, maps, g, partial, slice_len)); break;
        case 8: MG_TRY(launch_tma<8>(d, grid, smem, maps, g, partial, slice_len)); break;
        default: MG_TRY(launch_tma<16>(d, grid, smem, maps, g, partial, slice_len)); break;
    }
    return MG_OK;
}

// The cluster path: A K-major with 16-byte rows, B with 16-byte rows; k split so that the
// clusters fill the GPU about twice over (two CTAs per SM), at most 8 CTAs per cluster.
bool gemv_cluster_eligible(const GemmArgs& g) {
    auto al = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    return !g.transpose_a && !g.transpose_b && g.k % 4 == 0 && g.n % 4 == 0 && al(g.a) && al(g.b) &&
           (!g.b2 || al(g.b2)) && g.k < (1ull << 31) && g.n < (1ull << 31);
}

mg_status gemv_cluster(Device* d, const GemmArgs& g) {
    const uint64_t col_tiles = (g.n + kCols - 1) / kCols;
    if (col_tiles > 0x7FFFFFFFull) return fail(MG_SHAPE_UNSUPPORTED, "gemv n %llu is too wide", (unsigned long long)g.n);
    const int terms = g.gated ? 2 : 1;
    const int mp = g.m <= 1 ? 1 : g.m <= 2 ? 2 : g.m <= 4 ? 4 : g.m <= 8 ? 8 : 16;
    const uint64_t per_sm = mp >= 16 ? 1 : mp == 1 ? 3 : 2;  // CTAs per SM the launch fills
    uint64_t splits = (uint64_t)d->sm_count * per_sm / (col_tiles * terms);
    const uint64_t max_splits = kMaxClusterCtas / terms;
    if (splits > max_splits) splits = max_splits;
    GemvClusterArgs p;
    p.out = g.out;
    p.addend = g.addend;
    p.addend_mode = g.addend_mode;
    p.m = g.m;
    p.n = g.n;
    p.k = g.k;
    p.terms = terms;
    gemv_slices(p, splits);
    p.b_early = g.b_stable ? 1 : 0;
    p.error = d->flags + 2;
    // Compact weights (every value exactly bfloat16) stream as their bfloat16 bits: B and, gated,
    // the up weight both, or neither.
    const bool h = g.b16[0] && (!g.gated || g.b16[1]);
    CUtensorMap maps[3];
    MG_TRY(gemv_a_map(&maps[0], g.a, g.m, g.k, (uint32_t)mp));
    if (h) {
        MG_TRY(gemv_map_compact(&maps[1], g.b16[0], g.k, g.n));
        if (g.gated) MG_TRY(gemv_map_compact(&maps[2], g.b16[1], g.k, g.n));
        else maps[2] = maps[1];
        switch (mp) {
            case 1: return launch_cluster<1, true>(d, p, col_tiles, maps);
            case 2: return launch_cluster<2, true>(d, p, col_tiles, maps);
            case 4: return launch_cluster<4, true>(d, p, col_tiles, maps);
            case 8: return launch_cluster<8, true>(d, p, col_tiles, maps);
            default: return launch_cluster<16, true>(d, p, col_tiles, maps);
        }
    }
    MG_TRY(gemv_map(&maps[1], g.b, g.k, g.n));
    if (g.gated) MG_TRY(gemv_map(&maps[2], g.b2, g.k, g.n));
    else maps[2] = maps[1];
    switch (mp) {
        case 1: return launch_cluster<1, false>(d, p, col_tiles, maps);
        case 2: return launch_cluster<2, false>(d, p, col_tiles, maps);
        case 4: return launch_cluster<4, false>(d, p, col_tiles, maps);
        case 8: return launch_cluster<8, false>(d, p, col_tiles, maps);
        default: return launch_cluster<16, false>(d, p, col_tiles, maps);
    }
}

bool gemv_tc_eligible(const GemmArgs& g);
mg_status gemv_tc(Device* d, const GemmArgs& g);

mg_status gemv(Device* d, const GemmArgs& g) {
    // From about eight rows the CUDA-core kernels are bound by FMA issue: the tensor cores
    // take those (gemv_tc.cu).
    if (gemv_tc_eligible(g)) return gemv_tc(d, g);
    if (gemv_cluster_eligible(g)) return gemv_cluster(d, g);
    uint64_t tma_slices = 0, tma_slice_len = 0;
    if (g.n <= (1ull << 31) && g.k <= (1ull << 31) && gemv_tma_plan(d, g, &tma_slices, &tma_slice_len))
        return gemv_tma(d, g, tma_slices, tma_slice_len);
    const uint64_t col_tiles = (g.n + kCols - 1) / kCols;
    // Enough slices of k for about four CTAs per SM, each slice a multiple of the rows the
    // warps consume per step and at most 512 rows (A's slice fits shared memory).
    const uint64_t ctas_wanted = (uint64_t)d->sm_count * 4 / (g.gated ? 2 : 1);
    uint64_t slices = (ctas_wanted + col_tiles - 1) / col_tiles;
    const uint64_t step = kWarps * kRowsInFlight;
    uint64_t slice_len = (g.k + slices - 1) / slices;
    slice_len = ((slice_len + step - 1) / step) * step;
    if (slice_len > 512) slice_len = 512;
    if (slice_len < step) slice_len = step;
    slices = (g.k + slice_len - 1) / slice_len;
    if (slices == 0) slices = 1;
    const int mp = g.m <= 1 ? 1 : g.m <= 2 ? 2 : g.m <= 4 ? 4 : g.m <= 8 ? 8 : 16;
    const size_t smem = ((size_t)mp * slice_len + kWarps * kCols) * sizeof(float);
    const int zs = g.gated ? 2 : 1;
    float* partial = nullptr;
    MG_TRY(scratch(d, 0, (size_t)zs * slices * g.m * g.n * sizeof(float), (void**)&partial));
    dim3 grid((unsigned)col_tiles, (unsigned)slices, (unsigned)zs);
    switch (mp) {
        case 1: launch_partial<1>(d, grid, smem, g, partial, slice_len); break;
        case 2: launch_partial<2>(d, grid, smem, g, partial, slice_len); break;
        case 4: launch_partial<4>(d, grid, smem, g, partial, slice_len); break;
        case 8: launch_partial<8>(d, grid, smem, g, partial, slice_len); break;
        default: launch_partial<16>(d, grid, smem, g, partial, slice_len); break;
    }
    MG_TRY(launched(d, "gemv kernel launch"));
    uint64_t total = g.m * g.n;
    uint64_t blocks = (total + 255) / 256;
    if (blocks > (uint64_t)d->sm_count * 8) blocks = (uint64_t)d->sm_count * 8;
    enqueue(d, gemv_reduce_kernel, (unsigned)(blocks ? blocks : 1), 256, 0, partial, g.out, g.m, g.n, slices,
                                                                              g.addend, g.addend_mode, g.gated);
    return launched(d, "gemv reduce kernel launch");
}

}  // namespace k
}  // namespace mg

// =========================================================================================
// Fixed-workspace variant: the same two kernels, with the split-k partials kept in a
// workspace that lives inside the loaded library instead of coming from an allocator.
//
// Some callers cannot allocate device memory at the moment they multiply: a runtime whose
// device memory is already fully handed out under a fixed admission budget, or a
// latency-critical thread that must never enter the driver's allocator (which can block
// on a lock or on device-wide synchronisation).  For them, mg_matmul_gemv_fixed takes only
// caller-owned inputs and outputs and a stream, and keeps its partial sums in
// g_gemv_fixed_workspace below.
//
// That array is a file-scope __device__ variable: every GPU that loads this library holds
// one copy (MG_GEMV_FIXED_WORKSPACE_BYTES) until the process exits.  Host code cannot use
// its name as a device address, so the first call on each device looks the address up
// with cudaGetSymbolAddress while that device is current, and later calls reuse it.  All
// calls on a device share the one array and it keeps whatever the last call left there:
// every call overwrites each partial it reads, so nothing needs clearing, but calls that
// overlap on the GPU (different streams, no ordering between them) race on it.
// =========================================================================================
#include <mutex>

namespace {

constexpr uint64_t kFixedWorkspaceFloats = MG_GEMV_FIXED_WORKSPACE_BYTES / sizeof(float);
static __device__ __align__(256) float g_gemv_fixed_workspace[kFixedWorkspaceFloats];

struct FixedDevice {
    bool ready = false;
    float* workspace = nullptr;
    int sm_count = 0;
};
constexpr int kMaxFixedDevices = 64;
FixedDevice g_fixed_devices[kMaxFixedDevices];
std::mutex g_fixed_mutex;

// Looks up the workspace's device address and the SM count of `ordinal`, once.
mg_status fixed_setup(int ordinal, FixedDevice** out) {
    if (ordinal < 0 || ordinal >= kMaxFixedDevices)
        return mg::fail(MG_DEVICE_UNAVAILABLE, "device ordinal %d is outside 0..%d", ordinal, kMaxFixedDevices - 1);
    std::lock_guard<std::mutex> lock(g_fixed_mutex);
    FixedDevice& fd = g_fixed_devices[ordinal];
    if (!fd.ready) {
        int previous = 0;
        MG_CUDA(cudaGetDevice(&previous), "reading the current device");
        MG_CUDA(cudaSetDevice(ordinal), "selecting the device");
        void* ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&ptr, g_gemv_fixed_workspace);
        int sms = 0;
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, ordinal);
        cudaSetDevice(previous);
        if (e != cudaSuccess) return mg::from_cuda(e, "locating the fixed gemv workspace");
        fd.workspace = static_cast<float*>(ptr);
        fd.sm_count = sms;
        fd.ready = true;
    }
    *out = &fd;
    return MG_OK;
}

}  // namespace

extern "C" mg_status mg_matmul_gemv_fixed(int device_ordinal, void* stream, const float* a, const float* b,
                                          float* out, uint64_t m, uint64_t k, uint64_t n) {
    using namespace mg;
    if (!a || !b || !out) return fail(MG_INVALID_ARGUMENT, "null operand");
    if (m < 1 || m > kMaxRows) return fail(MG_SHAPE_UNSUPPORTED, "fixed-workspace gemv takes 1..16 rows, got %llu",
                                           (unsigned long long)m);
    if (k == 0 || n == 0 || n % 4 != 0)
        return fail(MG_SHAPE_UNSUPPORTED, "fixed-workspace gemv needs k > 0 and n a positive multiple of 4, got k %llu n %llu",
                    (unsigned long long)k, (unsigned long long)n);
    if ((reinterpret_cast<uintptr_t>(b) & 15) != 0)
        return fail(MG_LAYOUT_UNSUPPORTED, "fixed-workspace gemv needs b aligned to 16 bytes");
    FixedDevice* fd = nullptr;
    MG_TRY(fixed_setup(device_ordinal, &fd));
    // The split of k the allocating path would choose for this device.
    const uint64_t col_tiles = (n + kCols - 1) / kCols;
    const uint64_t ctas_wanted = (uint64_t)fd->sm_count * 4;
    uint64_t slices = (ctas_wanted + col_tiles - 1) / col_tiles;
    const uint64_t step = kWarps * kRowsInFlight;
    uint64_t slice_len = (k + slices - 1) / slices;
    slice_len = ((slice_len + step - 1) / step) * step;
    if (slice_len > 512) slice_len = 512;
    if (slice_len < step) slice_len = step;
    slices = (k + slice_len - 1) / slice_len;
    if (slices == 0) slices = 1;
    if (slices > 65535 || col_tiles > 0x7FFFFFFFull)
        return fail(MG_SHAPE_UNSUPPORTED, "fixed-workspace gemv shape exceeds the launch grid");
    const uint64_t need = slices * m * n;
    if (need > kFixedWorkspaceFloats)
        return fail(MG_SHAPE_UNSUPPORTED,
                    "fixed-workspace gemv needs %llu bytes of partial sums for m %llu k %llu n %llu; the fixed "
                    "workspace holds %llu bytes",
                    (unsigned long long)(need * sizeof(float)), (unsigned long long)m, (unsigned long long)k,
                    (unsigned long long)n, (unsigned long long)MG_GEMV_FIXED_WORKSPACE_BYTES);
    int previous = 0;
    MG_CUDA(cudaGetDevice(&previous), "reading the current device");
    MG_CUDA(cudaSetDevice(device_ordinal), "selecting the device");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int mp = m <= 1 ? 1 : m <= 2 ? 2 : m <= 4 ? 4 : m <= 8 ? 8 : 16;
    const size_t smem = ((size_t)mp * slice_len + kWarps * kCols) * sizeof(float);
    dim3 grid((unsigned)col_tiles, (unsigned)slices, 1);
    float* partial = fd->workspace;
    switch (mp) {
        case 1: gemv_partial_kernel<1><<<grid, kWarps * 32, smem, s>>>(a, b, nullptr, partial, m, n, k, slice_len, 0); break;
        case 2: gemv_partial_kernel<2><<<grid, kWarps * 32, smem, s>>>(a, b, nullptr, partial, m, n, k, slice_len, 0); break;
        case 4: gemv_partial_kernel<4><<<grid, kWarps * 32, smem, s>>>(a, b, nullptr, partial, m, n, k, slice_len, 0); break;
        case 8: gemv_partial_kernel<8><<<grid, kWarps * 32, smem, s>>>(a, b, nullptr, partial, m, n, k, slice_len, 0); break;
        default: gemv_partial_kernel<16><<<grid, kWarps * 32, smem, s>>>(a, b, nullptr, partial, m, n, k, slice_len, 0); break;
    }
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) {
        uint64_t blocks = (m * n + 255) / 256;
        if (blocks > (uint64_t)fd->sm_count * 8) blocks = (uint64_t)fd->sm_count * 8;
        gemv_reduce_kernel<<<(unsigned)(blocks ? blocks : 1), 256, 0, s>>>(partial, out, m, n, slices, nullptr, 0, 0);
        e = cudaGetLastError();
    }
    cudaSetDevice(previous);
    if (e != cudaSuccess) return from_cuda(e, "fixed-workspace gemv launch");
    return MG_OK;
}
