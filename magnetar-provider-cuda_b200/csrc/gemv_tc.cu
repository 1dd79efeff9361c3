// f32 matmul for a few rows (the decode side, 8 <= M <= 16) on the 5th-generation tensor cores,
// with B streamed from HBM exactly once.
//
// The CUDA-core few-row path (gemv.cu) spends two FLOPs of FMA issue per weight value per row:
// from about eight rows up it is bound by instruction issue, not by reading B.  Here the MMA is
// turned around so that the weight is the 128-row operand and the activation rows are the
// MMA's N: D[n][m] = sum_k B[k][n] * A[m][k].  A raw stage is B's [64 k][128 n] as it lies (one
// unswizzled TMA box) and A's [16][64].  Each operand enters as two tf32 terms (3xTF32, the f32
// contract): eight converter warps split the weight -- each thread its column n over 32 k --
// into hi (truncated to tf32) and lo = tf32(x - hi) and store both to tensor memory, where the
// MMA reads them as its A operand; A's hi and lo rows are stacked as the MMA's N = 32 in shared
// memory, so one thread issues W_lo [A_hi; A_lo] + W_hi [A_hi; A_lo] per k-step and the hi and lo
// rows of the accumulator are added at the end.  Shared memory carries only the raw stage and
// A's small terms.  The k slices of one 128-column tile (and, gated, the gate and up terms) form
// one thread-block cluster; each CTA stages its [16 x 128] partial, sends each band of rows to
// the CTA that owns it with one bulk copy, and owners add the partials in split order
// (deterministic), apply bias / residual / SwiGLU and write.
//
// Packed Q8_0 weights (tiled records) take a kernel of their own further down, on bf16 operands:
// every quant is exactly a bfloat16 value, so only the activations are split.
#include <cooperative_groups.h>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

#include "internal.h"
#include "sm100.cuh"

namespace mg {
namespace {

using namespace sm100;

constexpr int kTcCols = 128;     // columns of B per CTA: the MMA's M
constexpr int kTcK = 32;         // k per conversion group: one 128-byte swizzle row
constexpr int kTcRows = 16;      // the MMA's N: activation rows (zero past M)
constexpr int kAccs = 4;         // TMEM accumulators: k-step s of a group adds into accumulator s
constexpr int kConvThreads = 256;
constexpr int kMaxCluster = 16;  // non-portable cluster size (checked against the GPU at launch)
constexpr int kQ8Chunk = 128;    // k per tiled Q8_0 record

struct TcGemvShape {
    // A raw stage is 64 k: B's [64 k][128 n] as it lies (one unswizzled box, n contiguous), then
    // A's [16][64] as two 128-byte-swizzled [16][32] boxes (K-major, the MMA's B operand).
    static constexpr int kStageK = 2 * kTcK;
    static constexpr int kWRaw = kStageK * kTcCols * 4;   // 32 KB
    static constexpr int kAGroup = kTcRows * kTcK * 4;     // one [16][32] box: 2 KB
    static constexpr int kOffA = kWRaw;
    static constexpr int kRawStage = kOffA + 2 * kAGroup;  // 36 KB
    static constexpr int kRawStages = 5;                   // raw bytes in flight from HBM
    // A converted stage: the weight's hi / lo terms in tensor memory (64 + 64 columns of 128
    // lanes), A's hi / lo terms in shared memory as two K-major [32][32] tiles, one per 32 k:
    // rows 0-15 hi, rows 16-31 lo ([hi g0][lo g0][hi g1][lo g1]).
    static constexpr int kConvStage = 4 * kAGroup;         // 8 KB
    static constexpr int kConvStages = 3;
    static constexpr int kRing = kRawStages * kRawStage + kConvStages * kConvStage;
    static constexpr int kRecv = 32 * kTcCols * 4;         // the other CTAs' rows of this CTA's band
    static constexpr int kBars = 256;
    static constexpr int kSmem = kRing + kRecv + kBars + 1024;
    static constexpr int kThreads = 320;  // producer, MMA, 8 converter warps
    static constexpr uint32_t kTmemCols = 512;
    static constexpr int kN = 2 * kTcRows;                 // the MMA's N: A's hi rows, then its lo rows
    static constexpr uint32_t kWCol0 = kAccs * kN;         // accumulators first, then the weight stages
    static constexpr uint32_t kWStageCols = 2 * kStageK;   // hi then lo, one column per k
    static_assert(kRawStage % 1024 == 0 && kConvStage % 1024 == 0 && kOffA % 1024 == 0,
                  "swizzle atoms stay 1024-byte aligned");
    static_assert(kTcRows * kTcCols * 4 <= kRawStage, "the staged partial fits a drained raw stage");
    static_assert(kWCol0 + kConvStages * kWStageCols <= kTmemCols, "accumulators and weight stages fit");
    static_assert(kTcK / 8 == kAccs, "one accumulator per k-step of a group");
    static_assert(kSmem <= 227 * 1024, "shared memory budget");
};

struct GemvTcArgs {
    // Q8_0 B (tiled layout): quants / scales of B (and B2, gated), and k records per column tile
    const int8_t* quants[2];
    const float* scales[2];
    uint64_t chunks;
    float* out;
    const float* addend;
    int addend_mode;  // 0 none, 1 row [n], 2 full [m, n]
    uint64_t m, n, k;
    uint64_t slice_len;  // k rows per split (a multiple of kTcK)
    int splits;          // S; the cluster is (1, S, terms)
    int terms;           // 1, or 2 for gated (gate: z = 0, up: z = 1)
    int b_early;         // B does not depend on the preceding kernel: its first loads precede the wait
    int* error;
};

__device__ __forceinline__ float tf32_rna(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

// hi = x truncated to tf32 (nothing can overflow), lo = tf32(x - hi): exact to 2^-21 of x.
__device__ __forceinline__ void split_fast(float4 v, float4& hi, float4& lo) {
    hi = make_float4(__uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u), __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u),
                     __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u), __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u));
    lo = make_float4(tf32_rna(v.x - hi.x), tf32_rna(v.y - hi.y), tf32_rna(v.z - hi.z), tf32_rna(v.w - hi.w));
}

__global__ void __launch_bounds__(TcGemvShape::kThreads, 1)
    gemv_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                   const __grid_constant__ CUtensorMap map_b2, GemvTcArgs p) {
    using S = TcGemvShape;
    constexpr int kRawStages = S::kRawStages;
    constexpr int kConvStages = S::kConvStages;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* base_ptr = smem_raw + (base - raw);
    auto raw_stage = [&](int s) { return base + (uint32_t)(s * S::kRawStage); };
    auto conv_stage = [&](int c) { return base + (uint32_t)(kRawStages * S::kRawStage + c * S::kConvStage); };
    const uint32_t recv = base + S::kRing;
    const uint32_t bar_base = recv + S::kRecv;
    uint64_t* bars = reinterpret_cast<uint64_t*>(base_ptr + S::kRing + S::kRecv);
    auto raw_full = [&](int s) { return bar_base + 8u * s; };
    auto raw_empty = [&](int s) { return bar_base + 8u * (kRawStages + s); };
    auto conv_full = [&](int c) { return bar_base + 8u * (2 * kRawStages + c); };
    auto conv_empty = [&](int c) { return bar_base + 8u * (2 * kRawStages + kConvStages + c); };
    const uint32_t accum_bar = bar_base + 8u * (2 * kRawStages + 2 * kConvStages);
    const uint32_t recv_bar = accum_bar + 8u;
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(bars + 2 * kRawStages + 2 * kConvStages + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * kRawStages + 2 * kConvStages + 3);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int nc = p.splits * p.terms;
    const int rank = (int)cooperative_groups::this_cluster().block_rank();
    const int mb = ((int)p.m + nc - 1) / nc;  // activation rows each cluster CTA finishes
    const int my_lo = min((int)p.m, rank * mb), my_hi = min((int)p.m, my_lo + mb);
    const uint64_t n0 = (uint64_t)blockIdx.x * kTcCols;
    const int term = blockIdx.z;
    const CUtensorMap* map_w = term ? &map_b2 : &map_b;
    const uint64_t k0 = (uint64_t)blockIdx.y * p.slice_len;
    const uint64_t k1 = min(p.k, k0 + p.slice_len);
    const int num_kb = k1 > k0 ? (int)((k1 - k0 + S::kStageK - 1) / S::kStageK) : 0;  // raw stages

    // The producer's loads of raw stage i: B (the weight's [64 k][128 n]) arms the stage's barrier
    // for all its bytes; A's two boxes follow.  Past k (or n) the copies fill zeros.
    auto issue_w = [&](int i) {
        const int s = i % kRawStages;
        mbar_arrive_expect_tx(raw_full(s), (uint32_t)S::kRawStage);
        tma_load_2d(raw_stage(s), map_w, raw_full(s), (int)n0, (int)(k0 + (uint64_t)i * S::kStageK));
    };
    auto issue_a = [&](int i) {
        const int s = i % kRawStages;
        const int kx = (int)(k0 + (uint64_t)i * S::kStageK);
        tma_load_2d(raw_stage(s) + S::kOffA, &map_a, raw_full(s), kx, 0);
        tma_load_2d(raw_stage(s) + S::kOffA + S::kAGroup, &map_a, raw_full(s), kx + kTcK, 0);
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < kRawStages; s++) {
            mbar_init(raw_full(s), 1);
            mbar_init(raw_empty(s), kConvThreads / 32);
        }
        for (int c = 0; c < kConvStages; c++) {
            mbar_init(conv_full(c), kConvThreads / 32);
            mbar_init(conv_empty(c), 1);
        }
        mbar_init(accum_bar, 1);
        mbar_init(recv_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
        // The other CTAs' rows of this CTA's band, one bulk copy from each.
        mbar_arrive_expect_tx(recv_bar, (uint32_t)((nc - 1) * (my_hi - my_lo) * kTcCols * 4));
        if (p.b_early)
            for (int i = 0; i < min(kRawStages, num_kb); i++) issue_w(i);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32((const void*)tmem_slot), S::kTmemCols);
        tmem_relinquish();
    }
    cluster_arrive();  // phase 1: every receive barrier of the cluster is armed
    pdl_enter();
    if (threadIdx.x == 0) {
        for (int i = 0; i < min(kRawStages, num_kb); i++) {
            if (!p.b_early) issue_w(i);
            issue_a(i);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---- TMA producer: refills a raw stage once the converters have read it ------------
        if (lane == 0) {
            for (int i = kRawStages; i < num_kb; i++) {
                const int s = i % kRawStages;
                if (!mbar_wait(raw_empty(s), ((uint32_t)(i / kRawStages) & 1u) ^ 1u)) {
                    *abort_flag = 1;
                    atomicExch(p.error, 1);
                    break;
                }
                if (*abort_flag) break;
                issue_w(i);
                issue_a(i);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---- MMA issuer: D[128 n][16 m] += W_lo A_hi + W_hi A_lo + W_hi A_hi --------------------
        if (lane == 0) {
            // the weight terms from tensor memory (its n in the lanes, k along the columns), A's
            // terms K-major from shared memory
            constexpr uint32_t idesc = idesc_tf32(kTcCols, S::kN);
            bool ok = true;
            for (int i = 0; i < num_kb; i++) {
                const int c = i % kConvStages;
                if (!mbar_wait(conv_full(c), (uint32_t)(i / kConvStages) & 1u) || *abort_flag) {
                    *abort_flag = 1;
                    atomicExch(p.error, 1);
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t cs = conv_stage(c);
                const uint32_t tw = tmem + S::kWCol0 + (uint32_t)c * S::kWStageCols;
#pragma unroll
                for (int g = 0; g < 2; g++) {
#pragma unroll
                    for (int kk = 0; kk < kTcK / 8; kk++) {
                        const uint32_t whi = tw + (uint32_t)(g * kTcK + kk * 8), wlo = whi + S::kStageK;
                        // A's hi and lo rows together: the MMA's N = 32
                        const uint64_t da = desc_k_sw128(cs + (uint32_t)(g * 2 * S::kAGroup)) + (uint64_t)((kk * 32) >> 4);
                        // four accumulators, one per k-step of a group: four independent chains;
                        // W_lo (A_hi + A_lo) + W_hi (A_hi + A_lo), the hi and lo rows added at the end
                        const uint32_t acc = tmem + (uint32_t)(kk * S::kN);
                        mma_tf32_ts(acc, wlo, da, idesc, (i > 0 || g > 0) ? 1u : 0u);
                        mma_tf32_ts(acc, whi, da, idesc, 1u);
                    }
                }
                tc_commit(conv_empty(c));  // frees the converted terms once these MMAs have read them
            }
            if (ok && num_kb > 0) tc_commit(accum_bar);
            else mbar_arrive(accum_bar);  // release the epilogue
        }
        __syncwarp();
    } else {
        // ---- warps 2..9: split each raw stage into hi / lo terms: the weight's into tensor
        //      memory (row n of this warp's lane quarter, one k half), A's into shared memory ------
        const int t = threadIdx.x - 64;
        const int q = warp % 4, hp = (warp - 2) / 4;
        const int n = q * 32 + lane;
        for (int i = 0; i < num_kb; i++) {
            const int s = i % kRawStages;
            bool ok = mbar_wait(raw_full(s), (uint32_t)(i / kRawStages) & 1u);
            const uint32_t rs = raw_stage(s);
            const int c = i % kConvStages;
            ok = mbar_wait(conv_empty(c), ((uint32_t)(i / kConvStages) & 1u) ^ 1u) && ok;
            if (!ok) {
                *abort_flag = 1;
                atomicExch(p.error, 1);  // still arrive below so that no one waits for this thread
            }
            tc_fence_after();  // the MMAs that read these tensor-memory columns before have completed
            const uint32_t cs = conv_stage(c);
            const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + S::kWCol0 + (uint32_t)c * S::kWStageCols +
                                (uint32_t)(32 * hp);
#pragma unroll
            for (int h = 0; h < 2; h++) {
                // k rows 32 hp + 16 h .. + 15 of this thread's column n: one 4-byte load per row
                // (a warp reads 128 contiguous bytes of each row)
                float x[16];
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    const uint32_t row = (uint32_t)(32 * hp + 16 * h + j);
                    asm volatile("ld.shared::cta.f32 %0, [%1];" : "=f"(x[j]) : "r"(rs + row * (kTcCols * 4) + (uint32_t)n * 4));
                }
                uint32_t hv[16], lv[16];
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    const float hi = __uint_as_float(__float_as_uint(x[j]) & 0xFFFFE000u);
                    hv[j] = __float_as_uint(hi);
                    lv[j] = __float_as_uint(tf32_rna(x[j] - hi));
                }
                tmem_st16(ta + (uint32_t)(16 * h), hv);
                tmem_st16(ta + S::kStageK + (uint32_t)(16 * h), lv);
            }
            {
                // A's two [16][32] boxes: the same swizzled layout in the hi rows and the lo rows
                // (16 rows are two whole 8-row swizzle atoms)
                const uint32_t off = (uint32_t)t * 16;
                const uint32_t g = off / S::kAGroup, o = off % S::kAGroup;
                float4 hi4, lo4;
                split_fast(lds4(rs + S::kOffA + off), hi4, lo4);
                sts4(cs + g * 2 * S::kAGroup + o, hi4.x, hi4.y, hi4.z, hi4.w);
                sts4(cs + g * 2 * S::kAGroup + S::kAGroup + o, lo4.x, lo4.y, lo4.z, lo4.w);
            }
            tc_wait_st();         // the weight terms are in the tensor memory
            fence_proxy_async();  // the generic-proxy writes become visible to tcgen05.mma
            tc_fence_before();
            mbar_arrive_warp(conv_full(c));
            mbar_arrive_warp(raw_empty(s));
            if (__any_sync(0xffffffffu, *abort_flag)) break;
        }
    }
    bool acc_ready = false;
    if (warp >= 2 && warp < 6) {
        const bool waited = mbar_wait(accum_bar, 0);
        if (!waited) atomicExch(p.error, 1);
        // tcgen05.ld is warp-collective: the whole warp reads the accumulator or none of it.
        acc_ready = __all_sync(0xffffffffu, waited && !*abort_flag && num_kb > 0);
    }
    // ---- stage this CTA's partial as [16 m][128 n] in the drained first raw stage ----------------
    float* staged = reinterpret_cast<float*>(base_ptr + (raw_stage(0) - base));
    if (warp >= 2 && warp < 6) {
        tc_fence_after();
        const int q = warp % 4;
        const int n = q * 32 + lane;
        float v[16];
#pragma unroll
        for (int j = 0; j < 16; j++) v[j] = 0.0f;
        if (acc_ready) {
            // the accumulators added in order, each row's hi and lo column together (deterministic)
#pragma unroll
            for (int a = 0; a < kAccs; a++) {
                float w[32];
                tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(a * S::kN), w);
                tc_wait_ld();
#pragma unroll
                for (int j = 0; j < 16; j++) v[j] += w[j] + w[16 + j];
            }
        }
#pragma unroll
        for (int j = 0; j < kTcRows; j++) staged[j * kTcCols + n] = v[j];
        fence_proxy_async();  // the staged rows are read by bulk copies next
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, S::kTmemCols);
    }
    // ---- exchange: each band of rows to the CTA that owns it ------------------------------------
    cluster_wait();  // phase 1
    {
        const int o = (int)threadIdx.x - 64;  // one issuing thread per destination
        if (o >= 0 && o < nc && o != rank) {
            const int lo = min((int)p.m, o * mb), hi = min((int)p.m, lo + mb);
            if (hi > lo)
                bulk_copy_to_cluster(mapa(recv + (uint32_t)(rank * mb * kTcCols * 4), (uint32_t)o),
                                     raw_stage(0) + (uint32_t)(lo * kTcCols * 4), (uint32_t)((hi - lo) * kTcCols * 4),
                                     mapa(recv_bar, (uint32_t)o));
        }
    }
    if (!mbar_wait(recv_bar, 0)) atomicExch(p.error, 1);
    cluster_arrive();  // phase 2: every copy into this CTA has landed
    // ---- finish this CTA's rows: splits in order, per term ---------------------------------------
    const float* recvf = reinterpret_cast<const float*>(base_ptr + S::kRing);
    for (int e = (int)threadIdx.x; e < (my_hi - my_lo) * kTcCols; e += blockDim.x) {
        const int r = my_lo + e / kTcCols, c = e % kTcCols;
        const uint64_t col = n0 + (uint64_t)c;
        if (col >= p.n) continue;
        auto from = [&](int src) {
            return src == rank ? staged[r * kTcCols + c] : recvf[(src * mb + (r - my_lo)) * kTcCols + c];
        };
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

// ---- packed Q8_0 with bf16 operands -------------------------------------------------------------
// Every int8 quant is exactly a bfloat16 value, so the weight enters the MMA as it is stored -- one
// bf16 term, no split -- and only the activations are split, into three bf16 terms h + m + l
// (h the value truncated to bf16, m = bf16(x - h), l = bf16(x - h - m): within 2^-24 of x).  The
// three terms are stacked as the MMA's N = 48 (rows 0-15, 16-31, 32-47), so one kind::f16 MMA per
// 16 k reads the weight tile once for all of them.  A Q8_0 block's scale multiplies its 32 k only,
// so each block accumulates into its own TMEM slot (48 columns); four scaler warps read a record's
// four finished slots, add each slot's three terms, and fold it into their registers as
// sum += scale * block_sum -- the reference's per-block sum times the block's scale
// (src/kernels.cu:283-348).
//
// The unit of work is one raw stage, half a tiled record (128 columns x 128 k): it is converted
// as a whole and its eight MMAs are issued together, so each stage costs one pass of barrier
// hand-offs (raw -> converters -> MMA -> scalers).  The converted weight goes to tensor memory
// (tcgen05.st), where the MMA reads it as its A operand: shared memory then carries only the raw
// stage (written by the copy engine, read once by the converters) and the small activation tile,
// not a second and third pass over the widened weight.
constexpr int kQbSlots = 8;          // TMEM block slots of 48 columns: two stages' four blocks
constexpr int kQbN = 3 * kTcRows;    // the MMA's N: three activation terms of 16 rows

struct QbShape {
    static constexpr int kWRaw = kTcCols * kQ8Chunk;   // quants of 128 columns x 128 k
    static constexpr int kScales = kTcCols * 4 * 4;    // their [128][4] scales
    static constexpr int kOffA = kWRaw + kScales;
    static constexpr int kARaw = kTcRows * kTcK * 4 * 4;  // A's [16][128] as four [16][32] boxes
    static constexpr int kRawStage = kOffA + kARaw;       // 26 KB
    static constexpr int kRawStages = 4;
    // a converted stage: the weight's [128 n][128 k] bf16 in tensor memory (64 columns), the three
    // activation terms' [48][128] bf16 in shared memory, K-major, 128-byte swizzled, as two 64-k
    // atom columns
    static constexpr int kBAtom = kQbN * 128;             // [48 rows][64 k] bf16: 6 KB
    static constexpr int kConvStage = 2 * kBAtom;
    static constexpr int kConvStages = 2;
    static constexpr int kRing = kRawStages * kRawStage + kConvStages * kConvStage;
    static constexpr int kMaxCluster = 8;              // 8 CTAs' bands of 16 rows: at most 23 rows received
    static constexpr int kRecv = 24 * kTcCols * 4;
    static constexpr int kBars = 512;
    static constexpr int kSmem = kRing + kRecv + kBars + 1024;
    static constexpr int kThreads = 448;  // producer, MMA, 4 scaler warps, 8 converter warps
    static constexpr uint32_t kTmemCols = 512;
    static constexpr uint32_t kWCol0 = 2 * 4 * kQbN;     // weight stages after the block slots: column 384
    static constexpr uint32_t kWStageCols = kQ8Chunk / 2;  // 64
    static_assert(kRawStage % 1024 == 0 && kConvStage % 1024 == 0 && kOffA % 1024 == 0 && kBAtom % 1024 == 0,
                  "swizzle atoms aligned");
    static_assert(kTcRows * kTcCols * 4 <= kConvStage, "the staged partial fits a drained conversion buffer");
    static_assert(kWCol0 + kConvStages * kWStageCols <= kTmemCols, "slots and weight stages fit the tensor memory");
    static_assert(kSmem <= 227 * 1024, "shared memory budget");
};

__device__ __forceinline__ uint32_t bf16x2_rn(float lo, float hi) {
    const __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&b);
}

__global__ void __launch_bounds__(QbShape::kThreads, 1)
    gemv_tc_q8b_kernel(const __grid_constant__ CUtensorMap map_a, GemvTcArgs p) {
    using S = QbShape;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* base_ptr = smem_raw + (base - raw);
    auto raw_stage = [&](int s) { return base + (uint32_t)(s * S::kRawStage); };
    auto conv_stage = [&](int c) { return base + (uint32_t)(S::kRawStages * S::kRawStage + c * S::kConvStage); };
    const uint32_t recv = base + S::kRing;
    const uint32_t bar_base = recv + S::kRecv;
    uint64_t* bars = reinterpret_cast<uint64_t*>(base_ptr + S::kRing + S::kRecv);
    constexpr int R = S::kRawStages, C = S::kConvStages;
    auto raw_full = [&](int s) { return bar_base + 8u * s; };
    auto raw_empty = [&](int s) { return bar_base + 8u * (R + s); };
    auto conv_full = [&](int c) { return bar_base + 8u * (2 * R + c); };
    auto conv_empty = [&](int c) { return bar_base + 8u * (2 * R + C + c); };
    auto acc_full = [&](int h) { return bar_base + 8u * (2 * R + 2 * C + h); };       // per half of the slots
    auto acc_empty = [&](int h) { return bar_base + 8u * (2 * R + 2 * C + 2 + h); };
    const uint32_t recv_bar = bar_base + 8u * (2 * R + 2 * C + 4);
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(bars + 2 * R + 2 * C + 5);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * R + 2 * C + 6);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int nc = p.splits * p.terms;
    const int rank = (int)cooperative_groups::this_cluster().block_rank();
    const int mb = ((int)p.m + nc - 1) / nc;
    const int my_lo = min((int)p.m, rank * mb), my_hi = min((int)p.m, my_lo + mb);
    const uint64_t n0 = (uint64_t)blockIdx.x * kTcCols;
    const int term = blockIdx.z;
    const int8_t* quants = term ? p.quants[1] : p.quants[0];
    const float* scales = term ? p.scales[1] : p.scales[0];
    const uint64_t k0 = (uint64_t)blockIdx.y * p.slice_len;
    const uint64_t k1 = min(p.k, k0 + p.slice_len);
    const int num_kb = k1 > k0 ? (int)((k1 - k0) / kQ8Chunk) : 0;  // raw stages (record halves)
    const uint64_t rec0 = (n0 >> 8) * p.chunks + k0 / kQ8Chunk;  // this CTA's first record
    const uint64_t half = n0 & 255;

    auto issue_w = [&](int i) {
        const int s = i % R;
        const uint32_t st = raw_stage(s);
        mbar_arrive_expect_tx(raw_full(s), (uint32_t)S::kRawStage);
        const uint64_t row0 = (rec0 + (uint64_t)i) * 256 + half;
        bulk_load(st, quants + row0 * kQ8Chunk, (uint32_t)S::kWRaw, raw_full(s));
        bulk_load(st + S::kWRaw, scales + row0 * 4, (uint32_t)S::kScales, raw_full(s));
    };
    auto issue_a = [&](int i) {
        const int s = i % R;
#pragma unroll
        for (int j = 0; j < 4; j++)
            tma_load_2d(raw_stage(s) + S::kOffA + (uint32_t)(j * kTcRows * kTcK * 4), &map_a, raw_full(s),
                        (int)(k0 + (uint64_t)i * kQ8Chunk + (uint64_t)j * kTcK), 0);
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < R; s++) {
            mbar_init(raw_full(s), 1);
            mbar_init(raw_empty(s), 8);  // the converter warps
        }
        for (int c = 0; c < C; c++) {
            mbar_init(conv_full(c), 8);
            mbar_init(conv_empty(c), 1);
        }
        for (int h = 0; h < 2; h++) {
            mbar_init(acc_full(h), 1);
            mbar_init(acc_empty(h), 4);  // the scaler warps
        }
        mbar_init(recv_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
        mbar_arrive_expect_tx(recv_bar, (uint32_t)((nc - 1) * (my_hi - my_lo) * kTcCols * 4));
        // a packed weight changes only by an upload, which synchronises: its loads may precede the wait
        for (int i = 0; i < min(R, num_kb); i++) issue_w(i);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32((const void*)tmem_slot), S::kTmemCols);
        tmem_relinquish();
    }
    cluster_arrive();  // phase 1: every receive barrier of the cluster is armed
    pdl_enter();
    if (threadIdx.x == 0)
        for (int i = 0; i < min(R, num_kb); i++) issue_a(i);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    float acc[kTcRows];
#pragma unroll
    for (int j = 0; j < kTcRows; j++) acc[j] = 0.0f;

    if (warp == 0) {
        // ---- producer: refills a raw stage once the converters have read it ---------------------
        if (lane == 0) {
            for (int i = R; i < num_kb; i++) {
                const int s = i % R;
                if (!mbar_wait(raw_empty(s), ((uint32_t)(i / R) & 1u) ^ 1u) || *abort_flag) {
                    *abort_flag = 1;
                    atomicExch(p.error, 1);
                    break;
                }
                issue_w(i);
                issue_a(i);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---- MMA issuer: stage i's blocks 4i .. 4i + 3 into slot half i % 2, two MMAs per block:
        //      D[slot] (+)= W (bf16) x [A_h; A_m; A_l]^T ------------------------------------------
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16(kTcCols, kQbN);
            for (int i = 0; i < num_kb; i++) {
                const int c = i % C, h = i % 2;
                if (!mbar_wait(conv_full(c), (uint32_t)(i / C) & 1u) ||
                    !mbar_wait(acc_empty(h), ((uint32_t)(i / 2) & 1u) ^ 1u) || *abort_flag) {
                    *abort_flag = 1;
                    atomicExch(p.error, 1);
                    break;
                }
                tc_fence_after();
                const uint32_t cs = conv_stage(c), wt = tmem + S::kWCol0 + (uint32_t)c * S::kWStageCols;
#pragma unroll
                for (int kk = 0; kk < kQ8Chunk / 16; kk++) {
                    const uint32_t koff = (uint32_t)((kk % 4) * 32);  // within the 64-k atom column
                    const uint64_t da = desc_k_sw128(cs + (uint32_t)(kk / 4) * S::kBAtom + koff);
                    mma_bf16_ts(tmem + (uint32_t)((4 * h + kk / 2) * kQbN), wt + (uint32_t)(8 * kk), da, idesc,
                                (uint32_t)(kk % 2));
                }
                tc_commit(acc_full(h));    // the stage's four block sums are complete
                tc_commit(conv_empty(c));  // and its conversion buffer is free
            }
        }
        __syncwarp();
    } else if (warp >= 6) {
        // ---- converters (8 warps): a whole raw stage per pass -----------------------------------
        const int t = threadIdx.x - 192;  // 0..255
        // weight row n (a lane of this warp's quarter of the tensor memory), k half hp
        const int n = (warp % 4) * 32 + lane, hp = (warp - 6) / 4;
        for (int i = 0; i < num_kb; i++) {
            const int s = i % R, c = i % C;
            bool ok = mbar_wait(raw_full(s), (uint32_t)(i / R) & 1u);
            ok = mbar_wait(conv_empty(c), ((uint32_t)(i / C) & 1u) ^ 1u) && ok;
            if (!ok) {
                *abort_flag = 1;
                atomicExch(p.error, 1);
            }
            tc_fence_after();  // the MMAs that read this stage's tensor-memory columns have completed
            const uint32_t rs = raw_stage(s), cs = conv_stage(c);
            // activations: row m = t / 16, k 8f .. 8f + 7 (f = t % 16) from the raw [16][32] f32 box
            // f / 4 (128-byte swizzle) -> bf16 chunk f of the three term rows m, 16 + m, 32 + m
            const int m = t >> 4, f = t & 15;
            float4 x0, x1;
            {
                const uint32_t box = rs + S::kOffA + (uint32_t)((f >> 2) * kTcRows * kTcK * 4);
                const int f0 = (f & 3) * 2;
                x0 = lds4(box + (uint32_t)(m * 128 + ((f0 ^ (m & 7)) * 16)));
                x1 = lds4(box + (uint32_t)(m * 128 + (((f0 + 1) ^ (m & 7)) * 16)));
            }
            // weight: 64 quants of row n (pieces 4hp .. 4hp + 3 of the record row, stored permuted)
            uint4 qv[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const uint32_t piece = (uint32_t)((4 * hp + u) ^ (n & 7));
                qv[u] = *reinterpret_cast<const uint4*>(base_ptr + (rs - base) + (uint32_t)n * kQ8Chunk + piece * 16);
            }
            {
                uint32_t th[4], tm[4], tl[4];
                auto terms3 = [&](float xa, float xb, int e) {
                    const float ha = __uint_as_float(__float_as_uint(xa) & 0xFFFF0000u);  // truncated: no overflow
                    const float hb = __uint_as_float(__float_as_uint(xb) & 0xFFFF0000u);
                    const float ra = xa - ha, rb = xb - hb;
                    const float ma = __bfloat162float(__float2bfloat16_rn(ra));
                    const float mb2 = __bfloat162float(__float2bfloat16_rn(rb));
                    th[e] = (__float_as_uint(ha) >> 16) | (__float_as_uint(hb) & 0xFFFF0000u);
                    tm[e] = bf16x2_rn(ma, mb2);
                    tl[e] = bf16x2_rn(ra - ma, rb - mb2);
                };
                terms3(x0.x, x0.y, 0);
                terms3(x0.z, x0.w, 1);
                terms3(x1.x, x1.y, 2);
                terms3(x1.z, x1.w, 3);
                const uint32_t bt = cs + (uint32_t)(f >> 3) * S::kBAtom;
                const uint32_t cc = (uint32_t)(f & 7);
                auto put_row = [&](uint32_t row, const uint32_t (&w)[4]) {
                    const uint32_t off = row * 128 + ((cc ^ (row & 7)) * 16);
                    asm volatile("st.shared::cta.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(bt + off), "r"(w[0]),
                                 "r"(w[1]), "r"(w[2]), "r"(w[3])
                                 : "memory");
                };
                put_row((uint32_t)m, th);
                put_row((uint32_t)(kTcRows + m), tm);
                put_row((uint32_t)(2 * kTcRows + m), tl);
            }
            {
                // two quants -> two bf16 exactly: 0x43 | q & 0x7F is 128 + (q & 0x7F), 0x43 | q & 0x80
                // is 128 or 256 by the sign bit; their difference is q
                auto wid2 = [](uint32_t w, uint32_t sel) {
                    const uint32_t y = __byte_perm(w, 0x43u, sel);
                    uint32_t r;
                    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(y & 0xFF7FFF7Fu), "r"(y & 0xFF80FF80u));
                    return r;
                };
                // k = 64hp + 16u + e of the stage -> column 32hp + 8u + e / 2 of its tensor-memory stage
                const uint32_t wt = tmem + ((uint32_t)((warp % 4) * 32) << 16) + S::kWCol0 +
                                    (uint32_t)c * S::kWStageCols + (uint32_t)(32 * hp);
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const uint32_t w[8] = {wid2(qv[u].x, 0x4140u), wid2(qv[u].x, 0x4342u), wid2(qv[u].y, 0x4140u),
                                           wid2(qv[u].y, 0x4342u), wid2(qv[u].z, 0x4140u), wid2(qv[u].z, 0x4342u),
                                           wid2(qv[u].w, 0x4140u), wid2(qv[u].w, 0x4342u)};
                    tmem_st8(wt + (uint32_t)(8 * u), w);
                }
            }
            tc_wait_st();
            fence_proxy_async();  // the activation tile's generic-proxy writes become visible to the MMA
            tc_fence_before();
            mbar_arrive_warp(conv_full(c));
            mbar_arrive_warp(raw_empty(s));
            if (__any_sync(0xffffffffu, *abort_flag)) break;
        }
    } else {
        // ---- warps 2..5: fold each stage's four block slots into registers: sum += scale * block --
        // A stage's four scales per column are fetched one stage ahead, so their load latency stays
        // off the chain of slot waits.
        const int q = warp % 4, n = q * 32 + lane;
        bool failed = false;
        auto scale4 = [&](int r) {
            return __ldg(reinterpret_cast<const float4*>(scales + ((rec0 + (uint64_t)r) * 256 + half + n) * 4));
        };
        float4 sc_nxt = num_kb > 0 ? scale4(0) : make_float4(0.f, 0.f, 0.f, 0.f);
        for (int i = 0; i < num_kb; i++) {
            const int h = i % 2;
            const float4 sc = sc_nxt;
            if (i + 1 < num_kb) sc_nxt = scale4(i + 1);
            if (!failed && !mbar_wait(acc_full(h), (uint32_t)(i / 2) & 1u)) failed = true;
            failed = __any_sync(0xffffffffu, failed);
            if (!failed) {
                tc_fence_after();
                const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(4 * h * kQbN);
#pragma unroll
                for (int blk = 0; blk < 4; blk++) {
                    float v[kQbN];
                    tmem_ld16(ta + (uint32_t)(blk * kQbN), v);
                    tmem_ld16(ta + (uint32_t)(blk * kQbN + 16), v + 16);
                    tmem_ld16(ta + (uint32_t)(blk * kQbN + 32), v + 32);
                    tc_wait_ld();
                    const float scb = blk == 0 ? sc.x : blk == 1 ? sc.y : blk == 2 ? sc.z : sc.w;
#pragma unroll
                    for (int r = 0; r < kTcRows; r++)
                        acc[r] = fmaf(scb, (v[r] + v[kTcRows + r]) + v[2 * kTcRows + r], acc[r]);
                }
            }
            tc_fence_before();
            mbar_arrive_warp(acc_empty(h));
        }
        if (failed) {
            *abort_flag = 1;
            atomicExch(p.error, 1);
        }
    }
    // ---- stage this CTA's partial as [16 m][128 n] in the drained first conversion buffer ------
    tc_fence_before();
    __syncthreads();
    float* staged = reinterpret_cast<float*>(base_ptr + (conv_stage(0) - base));
    if (warp >= 2 && warp < 6) {
        const int n = (warp % 4) * 32 + lane;
#pragma unroll
        for (int j = 0; j < kTcRows; j++) staged[j * kTcCols + n] = *abort_flag ? 0.0f : acc[j];
        fence_proxy_async();  // the staged rows are read by bulk copies next
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, S::kTmemCols);
    }
    // ---- exchange: each band of rows to the CTA that owns it ------------------------------------
    cluster_wait();  // phase 1
    {
        const int o = (int)threadIdx.x - 64;
        if (o >= 0 && o < nc && o != rank) {
            const int lo = min((int)p.m, o * mb), hi = min((int)p.m, lo + mb);
            if (hi > lo)
                bulk_copy_to_cluster(mapa(recv + (uint32_t)(rank * mb * kTcCols * 4), (uint32_t)o),
                                     conv_stage(0) + (uint32_t)(lo * kTcCols * 4), (uint32_t)((hi - lo) * kTcCols * 4),
                                     mapa(recv_bar, (uint32_t)o));
        }
    }
    if (!mbar_wait(recv_bar, 0)) atomicExch(p.error, 1);
    cluster_arrive();  // phase 2: every copy into this CTA has landed
    const float* recvf = reinterpret_cast<const float*>(base_ptr + S::kRing);
    for (int e = (int)threadIdx.x; e < (my_hi - my_lo) * kTcCols; e += blockDim.x) {
        const int r = my_lo + e / kTcCols, c = e % kTcCols;
        const uint64_t col = n0 + (uint64_t)c;
        if (col >= p.n) continue;
        auto from = [&](int src) {
            return src == rank ? staged[r * kTcCols + c] : recvf[(src * mb + (r - my_lo)) * kTcCols + c];
        };
        float g = 0.0f;
        for (int s2 = 0; s2 < p.splits; s2++) g += from(s2);
        float v;
        if (p.terms == 2) {
            float u = 0.0f;
            for (int s2 = 0; s2 < p.splits; s2++) u += from(p.splits + s2);
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

PFN_cuTensorMapEncodeTiled_v12000 tc_gemv_encode_fn() {
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

// Row-major f32 [rows, cols], box [box_rows x 32 columns], zero past the edges; 128-byte swizzle
// (a K-major operand: 16-byte granules) or, `mn`, 128-byte swizzle in 32-byte granules (an
// MN-major tf32 operand).
// A [rows, cols] f32 matrix in boxes of [box_rows][32] with 128-byte swizzling, or -- plain_cols
// > 0 -- of [box_rows][plain_cols] as it lies (no swizzle).
mg_status tc_gemv_map(CUtensorMap* map, const float* ptr, uint64_t rows, uint64_t cols, uint32_t box_rows,
                      uint32_t plain_cols = 0) {
    auto fn = tc_gemv_encode_fn();
    if (!fn) return fail(MG_DRIVER_FAILED, "the driver does not provide cuTensorMapEncodeTiled");
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols * sizeof(float)};
    cuuint32_t box[2] = {plain_cols ? plain_cols : 32u, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ptr), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, plain_cols ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(MG_DRIVER_FAILED, "encoding a TMA descriptor failed (CUresult %d)", (int)r);
    return MG_OK;
}

// The fewest rows that take the f32 path (MAGNETAR_CUDA_FEWROW_TC: a row count, or 0 to leave
// the few-row matmul on the CUDA cores), and the packed Q8_0 path (MAGNETAR_CUDA_FEWROW_TC_Q8).
int env_min_rows(const char* name, int dflt) {
    const char* e = getenv(name);
    if (!e || !*e) return dflt;
    const int x = atoi(e);
    return x <= 0 ? kTcRows + 1 : x;
}
// Defaults from measurement at N = K = 4096 (six weights back to back): packed Q8_0 takes 11.5 -
// 11.9 us here for 1 - 16 rows, on the CUDA cores 8.4 / 9.7 / 13.6 / 20.4 us for 1 / 2 / 4 / 6 rows
// (61 us at 16); f32 takes 18.9 - 19.8 us here for 2 - 16 rows against 13.4 / 14.1 / 14.9 / 19.4 us
// on the CUDA cores for 2 / 4 / 8 / 16 rows -- the f32 form stays off: its pace is one
// converter -> MMA hand-off per 64 k (about 1 us per stage per CTA), not HBM.
int tc_min_rows() {
    static int v = env_min_rows("MAGNETAR_CUDA_FEWROW_TC", kTcRows + 1);
    return v;
}
int tc_q8_min_rows() {
    static int v = env_min_rows("MAGNETAR_CUDA_FEWROW_TC_Q8", 3);
    return v;
}

mg_status launch_gemv_tc(Device* d, const k::GemmArgs& g) {
    using S = TcGemvShape;
    auto kernel = gemv_tc_kernel;
    const uint64_t col_tiles = (g.n + kTcCols - 1) / kTcCols;
    if (col_tiles > 0x7FFFFFFFull) return fail(MG_SHAPE_UNSUPPORTED, "gemv n %llu is too wide", (unsigned long long)g.n);
    const int terms = g.gated ? 2 : 1;
    constexpr uint64_t kStageK = (uint64_t)S::kStageK;
    const uint64_t kb = (g.k + kStageK - 1) / kStageK;
    uint64_t splits = (uint64_t)d->sm_count / (col_tiles * terms);
    if (splits > (uint64_t)(kMaxCluster / terms)) splits = kMaxCluster / terms;
    if (splits > kb) splits = kb;
    if (splits < 1) splits = 1;
    GemvTcArgs p;
    memset(&p, 0, sizeof p);
    p.out = g.out;
    p.addend = g.addend;
    p.addend_mode = g.addend_mode;
    p.m = g.m;
    p.n = g.n;
    p.k = g.k;
    p.terms = terms;
    p.b_early = g.b_stable ? 1 : 0;
    p.error = d->flags + 2;
    auto set_splits = [&](uint64_t sp) {
        p.slice_len = ((kb + sp - 1) / sp) * kStageK;
        p.splits = (int)((g.k + p.slice_len - 1) / p.slice_len);
        if (p.splits < 1) p.splits = 1;
    };
    set_splits(splits);
    static bool configured[64] = {false};
    if (!configured[d->ordinal & 63]) {
        MG_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmem),
                "configuring the tensor-core gemv kernel");
        MG_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1),
                "allowing the tensor-core gemv kernel clusters of up to 16");
        configured[d->ordinal & 63] = true;
    }
    // Clusters larger than 8 only where the GPU holds them (queried once per size); otherwise
    // fewer k splits.
    static int fits[kMaxCluster + 1] = {0};  // 1 fits, -1 does not
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
            if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &q) != cudaSuccess) {
                (void)cudaGetLastError();
                clusters = 0;
            }
            fits[nc] = clusters > 0 ? 1 : -1;
        }
        if (fits[nc] > 0) break;
        set_splits((uint64_t)p.splits - 1);
    }
    CUtensorMap maps[3];
    MG_TRY(tc_gemv_map(&maps[0], g.a, g.m, g.k, kTcRows));
    MG_TRY(tc_gemv_map(&maps[1], g.b, g.k, g.n, S::kStageK, kTcCols));
    if (g.gated) MG_TRY(tc_gemv_map(&maps[2], g.b2, g.k, g.n, S::kStageK, kTcCols));
    else maps[2] = maps[1];
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
    MG_CUDA(cudaLaunchKernelEx(&cfg, kernel, maps[0], maps[1], maps[2], p), "tensor-core gemv launch");
    return launched(d, "tensor-core gemv launch");
}

}  // namespace

namespace k {

bool gemv_tc_eligible(const GemmArgs& g) {
    auto al = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    return g.m >= (uint64_t)tc_min_rows() && g.m <= (uint64_t)kTcRows && !g.transpose_a && !g.transpose_b &&
           g.k % 4 == 0 && g.n % 4 == 0 && al(g.a) && al(g.b) && (!g.b2 || al(g.b2)) && !g.packed[0] &&
           !g.packed[1] && g.k < (1ull << 31) && g.n < (1ull << 31);
}
// (A compact weight takes this path too, reading its f32 values: its results stay bit-identical to
// the same values stored as f32, which take it as well.)

mg_status gemv_tc(Device* d, const GemmArgs& g) { return launch_gemv_tc(d, g); }

// Every B a tiled packed Q8_0 weight (transposed storage, k a multiple of 128), A K-major with
// 16-byte rows.
bool gemv_tc_q8_eligible(const GemmArgs& g) {
    const int terms = g.gated ? 2 : 1;
    for (int t = 0; t < terms; t++)
        if (!g.packed[t] || !g.packed[t]->q8_tiled) return false;
    return g.m >= (uint64_t)tc_q8_min_rows() && g.m <= (uint64_t)kTcRows && !g.transpose_a && !g.transpose_b &&
           g.k % kQ8Chunk == 0 && g.k % 4 == 0 && (reinterpret_cast<uintptr_t>(g.a) & 15) == 0 && g.k < (1ull << 31) &&
           g.n < (1ull << 31);
}

mg_status gemv_tc_q8(Device* d, const GemmArgs& g) {
    using S = QbShape;
    const uint64_t col_tiles = (g.n + kTcCols - 1) / kTcCols;
    if (col_tiles > 0x7FFFFFFFull) return fail(MG_SHAPE_UNSUPPORTED, "gemv n %llu is too wide", (unsigned long long)g.n);
    const int terms = g.gated ? 2 : 1;
    const uint64_t kb = g.k / kQ8Chunk;
    uint64_t splits = (uint64_t)d->sm_count / (col_tiles * terms);
    if (splits > (uint64_t)(S::kMaxCluster / terms)) splits = S::kMaxCluster / terms;
    if (splits > kb) splits = kb;
    if (splits < 1) splits = 1;
    GemvTcArgs p;
    memset(&p, 0, sizeof p);
    p.out = g.out;
    p.addend = g.addend;
    p.addend_mode = g.addend_mode;
    p.m = g.m;
    p.n = g.n;
    p.k = g.k;
    p.terms = terms;
    p.b_early = 1;
    p.error = d->flags + 2;
    for (int t = 0; t < 2; t++) {
        const Buffer* w = g.packed[t < terms ? t : 0];
        p.quants[t] = static_cast<const int8_t*>(w->ptr);
        p.scales[t] = w->q8_scales;
    }
    p.chunks = kb;
    auto set_splits = [&](uint64_t sp) {
        p.slice_len = ((kb + sp - 1) / sp) * kQ8Chunk;
        p.splits = (int)((g.k + p.slice_len - 1) / p.slice_len);
        if (p.splits < 1) p.splits = 1;
    };
    set_splits(splits);
    static bool configured[64] = {false};
    if (!configured[d->ordinal & 63]) {
        MG_CUDA(cudaFuncSetAttribute(gemv_tc_q8b_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmem),
                "configuring the packed tensor-core gemv kernel");
        MG_CUDA(cudaFuncSetAttribute(gemv_tc_q8b_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1),
                "allowing the packed tensor-core gemv kernel clusters of up to 16");
        configured[d->ordinal & 63] = true;
    }
    static int fits[kMaxCluster + 1] = {0};
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
            if (cudaOccupancyMaxActiveClusters(&clusters, gemv_tc_q8b_kernel, &q) != cudaSuccess) {
                (void)cudaGetLastError();
                clusters = 0;
            }
            fits[nc] = clusters > 0 ? 1 : -1;
        }
        if (fits[nc] > 0) break;
        set_splits((uint64_t)p.splits - 1);
    }
    CUtensorMap map_a;
    MG_TRY(tc_gemv_map(&map_a, g.a, g.m, g.k, kTcRows));
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
    MG_CUDA(cudaLaunchKernelEx(&cfg, gemv_tc_q8b_kernel, map_a, p), "packed tensor-core gemv launch");
    return launched(d, "packed tensor-core gemv launch");
}

}  // namespace k
}  // namespace mg
