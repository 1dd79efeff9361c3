// f32 matmul on the 5th-generation tensor cores: tcgen05 kind::tf32 MMAs accumulating in
// TMEM, operands staged in shared memory by TMA, 3xTF32 split precision.
//
// The reference runs every f32-weight matmul of M >= 64 on the CUDA cores
// (`matmul_split_k_tile_kernel`, src/kernels.cu:1643-1693) and keeps its tensor-core
// kernels (`mma.sync` bf16, src/tensor_kernels.cu:393-705) for bf16-exact weights.  Here:
//
//  1. A split pass writes each operand as two K-major tf32 terms, x = hi + lo with
//     hi = tf32(x) (rounded, truncated instead when rounding would overflow a finite
//     value to infinity) and lo = tf32(x - hi).  B (row-major [K, N]) is transposed to
//     [N, K] in the same pass, so both operands feed the MMA K-major.
//  2. The GEMM kernel: one 128 x BN output tile per CTA.  Warp 0 issues TMA loads of
//     A.hi, A.lo, B.hi, B.lo (32 k-columns = one 128-byte swizzle row per tile row) into a
//     STAGES-deep ring; warp 1 allocates TMEM and issues, per 8-wide k step, the three
//     products lo*hi + hi*lo + hi*hi into one f32 accumulator (the dropped lo*lo term is
//     below 2^-22 relative); warps 2-5 read the accumulator back with tcgen05.ld and apply
//     the addend (bias row / residual) or the SwiGLU gate before storing.
//  Error of each product is about 2^-22 relative, well inside the f32 contract's 1e-4
//  relative-L2 bound for matmul.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

#include "internal.h"
#include "sm100.cuh"

namespace mg {
namespace k {
bool gemv_eligible(const GemmArgs& g);
mg_status gemv(Device* d, const GemmArgs& g);
mg_status gemm_simt(Device* d, const GemmArgs& g);
}  // namespace k

namespace {

using namespace sm100;

constexpr int BM = 128;
constexpr int BK = 32;  // f32 k-columns per stage: one 128-byte swizzle row
constexpr int kThreadsTC = 192;
constexpr int kGroupM = 16;  // rasterisation: M-tiles walked together for L2 reuse

// ---- split pass ------------------------------------------------------------------------------
__device__ __forceinline__ float tf32_round(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
    float h = tf32_round(x);
    if (isinf(h) && !isinf(x)) h = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
    hi = h;
    lo = tf32_round(x - h);
}

// src [rows, k] (row stride ld) -> hi/lo [rows, kp], zero past k.
__global__ void __launch_bounds__(256) split_rows_kernel(const float* __restrict__ src, uint64_t ld, uint64_t rows,
                                                         uint64_t k, float* __restrict__ hi, float* __restrict__ lo,
                                                         uint64_t kp) {
    const uint64_t total = rows * kp;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t r = i / kp, c = i % kp;
        float h = 0.0f, l = 0.0f;
        if (c < k) split_tf32(src[r * ld + c], h, l);
        hi[i] = h;
        lo[i] = l;
    }
}

// src [r_count, c_count] row-major -> hi/lo [c_count, rp] with dst[c][r] = src[r][c].
__global__ void __launch_bounds__(256) split_transpose_kernel(const float* __restrict__ src, uint64_t r_count,
                                                              uint64_t c_count, float* __restrict__ hi,
                                                              float* __restrict__ lo, uint64_t rp) {
    __shared__ float tile[32][33];
    const uint64_t c0 = (uint64_t)blockIdx.x * 32, r0 = (uint64_t)blockIdx.y * 32;
    const int tx = threadIdx.x % 32, ty = threadIdx.x / 32;  // 32 x 8
    for (int j = ty; j < 32; j += 8) {
        const uint64_t r = r0 + j, c = c0 + tx;
        tile[j][tx] = (r < r_count && c < c_count) ? src[r * c_count + c] : 0.0f;
    }
    __syncthreads();
    for (int j = ty; j < 32; j += 8) {
        const uint64_t c = c0 + j, r = r0 + tx;
        if (c < c_count && r < rp) {
            float h, l;
            split_tf32(tile[tx][j], h, l);
            hi[c * rp + r] = h;
            lo[c * rp + r] = l;
        }
    }
}

// ---- the tensor-core GEMM ---------------------------------------------------------------------
struct TcParams {
    float* out;
    const float* addend;
    int addend_mode;
    int gated;
    uint64_t m, n, k;
    int tiles_m, tiles_n;
    int* error;  // device word set when a wait times out
};

template <int BN, int NB, int STAGES>
struct TcShape {
    static constexpr int kATile = BM * BK * 4;          // bytes of one A term tile
    static constexpr int kBTile = BN * BK * 4;          // bytes of one B term tile
    static constexpr int kStage = 2 * kATile + NB * 2 * kBTile;
    static constexpr int kSmem = STAGES * kStage + 1024 /* align */ + 256 /* barriers */;
    static constexpr uint32_t kTmemCols = NB * BN <= 32 ? 32 : NB * BN <= 64 ? 64 : NB * BN <= 128 ? 128 : NB * BN <= 256 ? 256 : 512;
};

template <int BN, int NB, int STAGES>
__global__ void __launch_bounds__(kThreadsTC, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap map_ahi, const __grid_constant__ CUtensorMap map_alo,
                   const __grid_constant__ CUtensorMap map_bhi, const __grid_constant__ CUtensorMap map_blo,
                   const __grid_constant__ CUtensorMap map_b2hi, const __grid_constant__ CUtensorMap map_b2lo,
                   TcParams p) {
    using S = TcShape<BN, NB, STAGES>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* base_ptr = smem_raw + (base - raw);
    const uint32_t bar_base = base + STAGES * S::kStage;
    uint64_t* bars = reinterpret_cast<uint64_t*>(base_ptr + STAGES * S::kStage);
    // bars[0..STAGES): full, [STAGES..2*STAGES): empty, [2*STAGES]: accumulator ready
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(bars + 2 * STAGES + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * STAGES + 2);
    (void)bars;
    auto full_bar = [&](int s) { return bar_base + 8u * s; };
    auto empty_bar = [&](int s) { return bar_base + 8u * (STAGES + s); };
    const uint32_t accum_bar = bar_base + 8u * (2 * STAGES);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

    // Grouped rasterisation of the 1-D grid over (tiles_m, tiles_n).
    const int tile = blockIdx.x;
    const int group_size = kGroupM * p.tiles_n;
    const int group = tile / group_size;
    const int first_m = group * kGroupM;
    const int rows_in_group = min(p.tiles_m - first_m, kGroupM);
    const int tm = first_m + (tile % group_size) % rows_in_group;
    const int tn = (tile % group_size) / rows_in_group;
    const int m0 = tm * BM, n0 = tn * BN;
    const int num_kb = (int)((p.k + BK - 1) / BK);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        mbar_init(accum_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tensormap(&map_ahi);
        prefetch_tensormap(&map_alo);
        prefetch_tensormap(&map_bhi);
        prefetch_tensormap(&map_blo);
        if (NB == 2) {
            prefetch_tensormap(&map_b2hi);
            prefetch_tensormap(&map_b2lo);
        }
    }
    if (warp == 1) {
        tmem_alloc(smem_u32((const void*)tmem_slot), S::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---- TMA producer --------------------------------------------------------------
        if (lane == 0) {
            for (int kb = 0; kb < num_kb; kb++) {
                const int s = kb % STAGES;
                const uint32_t phase = (uint32_t)(kb / STAGES) & 1u;
                if (!mbar_wait(empty_bar(s), phase ^ 1u)) {
                    *abort_flag = 1;
                    atomicExch(p.error, 1);
                    break;
                }
                if (*abort_flag) break;
                const uint32_t st = base + s * S::kStage;
                mbar_arrive_expect_tx(full_bar(s), S::kStage);
                const int kx = kb * BK;
                tma_load_2d(st, &map_ahi, full_bar(s), kx, m0);
                tma_load_2d(st + S::kATile, &map_alo, full_bar(s), kx, m0);
                tma_load_2d(st + 2 * S::kATile, &map_bhi, full_bar(s), kx, n0);
                tma_load_2d(st + 2 * S::kATile + S::kBTile, &map_blo, full_bar(s), kx, n0);
                if (NB == 2) {
                    tma_load_2d(st + 2 * S::kATile + 2 * S::kBTile, &map_b2hi, full_bar(s), kx, n0);
                    tma_load_2d(st + 2 * S::kATile + 3 * S::kBTile, &map_b2lo, full_bar(s), kx, n0);
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---- MMA issuer ----------------------------------------------------------------
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_tf32(BM, BN);
            bool ok = true;
            for (int kb = 0; kb < num_kb; kb++) {
                const int s = kb % STAGES;
                const uint32_t phase = (uint32_t)(kb / STAGES) & 1u;
                if (!mbar_wait(full_bar(s), phase)) {
                    *abort_flag = 1;
                    atomicExch(p.error, 1);
                    ok = false;
                    break;
                }
                if (*abort_flag) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t st = base + s * S::kStage;
                const uint64_t ahi = desc_k_sw128(st), alo = desc_k_sw128(st + S::kATile);
#pragma unroll
                for (int kk = 0; kk < BK / 8; kk++) {
                    const uint64_t koff = (uint64_t)((kk * 32) >> 4);  // 8 tf32 = 32 bytes
#pragma unroll
                    for (int z = 0; z < NB; z++) {
                        const uint32_t bt = st + 2 * S::kATile + z * 2 * S::kBTile;
                        const uint64_t bhi = desc_k_sw128(bt), blo = desc_k_sw128(bt + S::kBTile);
                        const uint32_t d = tmem + (uint32_t)(z * BN);
                        const uint32_t acc = (kb > 0 || kk > 0) ? 1u : 0u;
                        mma_tf32(d, alo + koff, bhi + koff, idesc, acc);
                        mma_tf32(d, ahi + koff, blo + koff, idesc, 1u);
                        mma_tf32(d, ahi + koff, bhi + koff, idesc, 1u);
                    }
                }
                tc_commit(empty_bar(s));  // frees the stage once these MMAs have read it
            }
            if (ok) tc_commit(accum_bar);
            else mbar_arrive(accum_bar);  // release the epilogue
        }
        __syncwarp();
    } else {
        // ---- epilogue: warps 2..5 own TMEM lane quarters (warp % 4) ----------------------
        const int q = warp % 4;
        const bool waited = mbar_wait(accum_bar, 0);
        if (!waited) atomicExch(p.error, 1);
        tc_fence_after();
        // tcgen05.ld is warp-collective: the whole warp reads the accumulator or none of it.
        const bool ready = __all_sync(0xffffffffu, waited && !*abort_flag);
        if (ready) {
            const uint64_t row = (uint64_t)m0 + q * 32 + lane;
            const bool row_ok = row < p.m;
            const bool vec = (p.n % 4 == 0) && ((reinterpret_cast<uintptr_t>(p.out) & 15) == 0) &&
                             (p.addend_mode != 2 || (reinterpret_cast<uintptr_t>(p.addend) & 15) == 0) &&
                             (p.addend_mode != 1 || (reinterpret_cast<uintptr_t>(p.addend) & 15) == 0);
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 32) {
                float v[32];
                tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, v);
                float u[32];
                if (NB == 2) tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(BN + c0), u);
                tc_wait_ld();
                if (!row_ok) continue;
                const uint64_t col0 = (uint64_t)n0 + c0;
                float* orow = p.out + row * p.n;
#pragma unroll
                for (int j = 0; j < 32; j++) {
                    float s = v[j];
                    if (NB == 2) {
                        s = (s * (1.0f / (1.0f + expf(-s)))) * u[j];
                    } else if (p.addend_mode == 1) {
                        if (col0 + j < p.n) s += p.addend[col0 + j];
                    } else if (p.addend_mode == 2) {
                        if (col0 + j < p.n) s += p.addend[row * p.n + col0 + j];
                    }
                    v[j] = s;
                }
                if (vec && col0 + 32 <= p.n) {
#pragma unroll
                    for (int j = 0; j < 32; j += 4)
                        *reinterpret_cast<float4*>(orow + col0 + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; j++)
                        if (col0 + j < p.n) orow[col0 + j] = v[j];
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, S::kTmemCols);
    }
}

// ---- host side ---------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// K-major [rows, kp] f32 matrix, box [box_rows, 32] with 128-byte swizzle.
mg_status make_map(CUtensorMap* map, const float* ptr, uint64_t rows, uint64_t kp, uint32_t box_rows) {
    auto fn = encode_fn();
    if (!fn) return fail(MG_DRIVER_FAILED, "the driver does not provide cuTensorMapEncodeTiled");
    cuuint64_t dims[2] = {kp, rows};
    cuuint64_t strides[1] = {kp * sizeof(float)};
    cuuint32_t box[2] = {BK, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ptr), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(MG_DRIVER_FAILED, "encoding a TMA descriptor failed (CUresult %d)", (int)r);
    return MG_OK;
}

inline unsigned grid_cap(const Device* d, uint64_t items) {
    uint64_t want = (items + 255) / 256, cap = (uint64_t)d->sm_count * 8;
    return (unsigned)(want < 1 ? 1 : want > cap ? cap : want);
}

// Writes the K-major hi/lo terms of an operand; `kmajor` says whether the stored matrix
// already has k contiguous ([rows, k]) or is [k, rows] and must be transposed.
mg_status split_operand(Device* d, const float* src, uint64_t rows, uint64_t k, bool kmajor, float* hi, float* lo,
                        uint64_t kp) {
    if (kmajor) {
        split_rows_kernel<<<grid_cap(d, rows * kp), 256, 0, d->stream>>>(src, k, rows, k, hi, lo, kp);
    } else {
        dim3 grid((unsigned)((rows + 31) / 32), (unsigned)((kp + 31) / 32));
        if (grid.y > 65535) return fail(MG_SHAPE_UNSUPPORTED, "matmul inner dimension %llu is too large", (unsigned long long)k);
        split_transpose_kernel<<<grid, 256, 0, d->stream>>>(src, k, rows, hi, lo, kp);
    }
    return launched(d, "operand split kernel launch");
}

template <int BN, int NB, int STAGES>
mg_status launch_tc(Device* d, const k::GemmArgs& g, const CUtensorMap* maps, int* err) {
    using S = TcShape<BN, NB, STAGES>;
    static bool configured[64] = {false};
    if (!configured[d->ordinal & 63]) {
        MG_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<BN, NB, STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmem),
                "configuring the tensor-core matmul");
        configured[d->ordinal & 63] = true;
    }
    TcParams p;
    p.out = g.out;
    p.addend = g.addend;
    p.addend_mode = g.addend_mode;
    p.gated = g.gated;
    p.m = g.m;
    p.n = g.n;
    p.k = g.k;
    p.tiles_m = (int)((g.m + BM - 1) / BM);
    p.tiles_n = (int)((g.n + BN - 1) / BN);
    p.error = err;
    const uint64_t tiles = (uint64_t)p.tiles_m * p.tiles_n;
    if (tiles > 0x7FFFFFFFull) return fail(MG_SHAPE_UNSUPPORTED, "matmul has too many output tiles");
    gemm_tc_kernel<BN, NB, STAGES><<<(unsigned)tiles, kThreadsTC, S::kSmem, d->stream>>>(
        maps[0], maps[1], maps[2], maps[3], maps[4], maps[5], p);
    return launched(d, "tensor-core matmul launch");
}

bool tensor_cores_enabled() {
    static int enabled = -1;
    if (enabled < 0) {
        const char* v = getenv("MAGNETAR_CUDA_TENSOR_CORES");
        enabled = (v && strcmp(v, "0") == 0) ? 0 : 1;
    }
    return enabled == 1;
}

}  // namespace

namespace k {

mg_status gemm_tc(Device* d, const GemmArgs& g) {
    const uint64_t kp = (g.k + 3) & ~3ull;  // TMA row strides are multiples of 16 bytes
    const int nb = g.gated ? 2 : 1;
    float *a_split = nullptr, *b_split = nullptr;
    MG_TRY(scratch(d, 1, 2 * g.m * kp * sizeof(float), (void**)&a_split));
    MG_TRY(scratch(d, 2, (size_t)nb * 2 * g.n * kp * sizeof(float), (void**)&b_split));
    float* ahi = a_split;
    float* alo = a_split + g.m * kp;
    // A is K-major unless transposed; B (row-major [K, N]) is K-major only when transposed.
    MG_TRY(split_operand(d, g.a, g.m, g.k, !g.transpose_a, ahi, alo, kp));
    float* bhi[2];
    float* blo[2];
    for (int z = 0; z < nb; z++) {
        bhi[z] = b_split + (size_t)z * 2 * g.n * kp;
        blo[z] = bhi[z] + g.n * kp;
        MG_TRY(split_operand(d, z ? g.b2 : g.b, g.n, g.k, g.transpose_b != 0, bhi[z], blo[z], kp));
    }
    constexpr int BN = 128;
    CUtensorMap maps[6];
    MG_TRY(make_map(&maps[0], ahi, g.m, kp, BM));
    MG_TRY(make_map(&maps[1], alo, g.m, kp, BM));
    MG_TRY(make_map(&maps[2], bhi[0], g.n, kp, BN));
    MG_TRY(make_map(&maps[3], blo[0], g.n, kp, BN));
    if (nb == 2) {
        MG_TRY(make_map(&maps[4], bhi[1], g.n, kp, BN));
        MG_TRY(make_map(&maps[5], blo[1], g.n, kp, BN));
    } else {
        maps[4] = maps[2];
        maps[5] = maps[3];
    }
    int* err = d->flags + 2;
    if (nb == 2) return launch_tc<BN, 2, 2>(d, g, maps, err);
    return launch_tc<BN, 1, 3>(d, g, maps, err);
}

mg_status gemm(Device* d, const GemmArgs& g) {
    if (g.m == 0 || g.n == 0) return MG_OK;
    if (g.k == 0) {
        // An empty inner dimension: every sum is 0 before the addend / gate.
        return gemm_simt(d, g);
    }
    if (gemv_eligible(g)) return gemv(d, g);
    if (tensor_cores_enabled() && g.m > 16) return gemm_tc(d, g);
    return gemm_simt(d, g);
}

}  // namespace k
}  // namespace mg
