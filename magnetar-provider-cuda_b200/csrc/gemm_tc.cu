// f32 matmul on the 5th-generation tensor cores: tcgen05 kind::tf32 MMAs accumulating in
// TMEM, operands staged in shared memory by TMA, 3xTF32 split precision.
//
// The reference runs every f32-weight matmul of M >= 64 on the CUDA cores
// (`matmul_split_k_tile_kernel`, src/kernels.cu:1643-1693) and keeps its tensor-core
// kernels (`mma.sync` bf16, src/tensor_kernels.cu:393-705) for bf16-exact weights.  Here each
// operand x enters the MMA as two tf32 terms, x = hi + lo with hi = tf32(x) (rounded;
// truncated instead when rounding would overflow a finite value to infinity) and
// lo = tf32(x - hi), and the kernel accumulates lo*hi + hi*lo + hi*hi in f32 TMEM -- the
// dropped lo*lo term is below 2^-22 relative, far inside the f32 contract's 1e-4 rel-L2.
//
// One CTA computes a 128 x BN output tile over a range of k:
//   warp 0      TMA producer: 32-column k-blocks (one 128-byte swizzle row per tile row) of
//               A and B into a STAGES-deep shared-memory ring;
//   warp 1      allocates TMEM and issues the MMAs (one thread), committing each stage back;
//   warps 2-9   (when A or B arrives as raw f32) split each raw tile into its hi/lo terms in
//               shared memory during the main loop, so no separate pass over the operand is
//               needed; afterwards warps 2-5 read the accumulator (tcgen05.ld) into the drained
//               shared-memory ring.
// When the output grid alone would leave SMs idle, k is split across the CTAs of a thread-block
// cluster; the partial tiles are then summed through distributed shared memory and every
// thread writes finished rows (bias / residual / SwiGLU applied) with coalesced stores.
// B comes either from a weight's prepared hi/lo form (built once, kept with the weight) or
// from a per-call split pass that also transposes it to K-major.
#include <cooperative_groups.h>
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

#include "internal.h"
#include "rope.cuh"
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
constexpr int BK = 32;       // f32 k-columns per stage: one 128-byte swizzle row
constexpr int kGroupM = 16;  // rasterisation: M-tiles walked together for L2 reuse
constexpr int kMaxSplits = 16;  // k splits of one tile: the CTAs of one (non-portable) cluster
constexpr int kConvThreads = 256;  // warps 2-9 split raw operand tiles during the main loop

// ---- operand split ----------------------------------------------------------------------------
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

__device__ __forceinline__ void split4(float4 v, float4& hi, float4& lo) {
    split_tf32(v.x, hi.x, lo.x);
    split_tf32(v.y, hi.y, lo.y);
    split_tf32(v.z, hi.z, lo.z);
    split_tf32(v.w, hi.w, lo.w);
}

// The in-kernel split of raw operand tiles (on the MMA's critical path): hi = x truncated to
// tf32 (no rounding, so nothing overflows), lo = tf32_rna(x - hi), which is exact to 2^-21 of
// x -- inside the f32 contract with room to spare, and three instructions per value.
__device__ __forceinline__ float4 trunc_tf32x4(float4 v) {
    return make_float4(__uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u),
                       __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u),
                       __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u),
                       __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u));
}
__device__ __forceinline__ void split4_fast(float4 v, float4& hi, float4& lo) {
    hi = trunc_tf32x4(v);
    lo = make_float4(tf32_round(v.x - hi.x), tf32_round(v.y - hi.y), tf32_round(v.z - hi.z), tf32_round(v.w - hi.w));
}

// Sets *flag (when not null) if any lane of the warp saw a nonzero lo term.  Every lane of
// the warp calls it once, after its loop.
__device__ __forceinline__ void note_lo(int* flag, bool nonzero) {
    if (!flag) return;
    if (__any_sync(0xffffffffu, nonzero) && (threadIdx.x & 31) == 0) atomicOr(flag, 1);
}

// src [rows, k] (row stride ld) -> hi/lo [rows, kp], zero past k.  16-byte vectors when the
// rows allow it.  `lo_nonzero` (optional): set when any lo term is nonzero.
__global__ void __launch_bounds__(256) split_rows_kernel(const float* __restrict__ src, uint64_t ld, uint64_t rows,
                                                         uint64_t k, float* __restrict__ hi, float* __restrict__ lo,
                                                         uint64_t kp, int vec, int* lo_nonzero) {
    pdl_enter();
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t t0 = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    bool nz = false;
    if (vec) {  // k == kp, k % 4 == 0, 16-byte aligned
        const uint64_t n4 = rows * kp / 4;
        const float4* s4 = reinterpret_cast<const float4*>(src);
        for (uint64_t i = t0; i < n4; i += stride) {
            float4 h, l;
            split4(s4[i], h, l);
            reinterpret_cast<float4*>(hi)[i] = h;
            reinterpret_cast<float4*>(lo)[i] = l;
            nz = nz || l.x != 0.0f || l.y != 0.0f || l.z != 0.0f || l.w != 0.0f;
        }
    } else {
        const uint64_t total = rows * kp;
        for (uint64_t i = t0; i < total; i += stride) {
            const uint64_t r = i / kp, c = i % kp;
            float h = 0.0f, l = 0.0f;
            if (c < k) split_tf32(src[r * ld + c], h, l);
            hi[i] = h;
            lo[i] = l;
            nz = nz || l != 0.0f;
        }
    }
    note_lo(lo_nonzero, nz);
}

// src [r_count, c_count] row-major -> hi/lo [c_count, rp] with dst[c][r] = src[r][c], through
// 64 x 64 shared-memory tiles.
__global__ void __launch_bounds__(256) split_transpose_kernel(const float* __restrict__ src, uint64_t r_count,
                                                              uint64_t c_count, float* __restrict__ hi,
                                                              float* __restrict__ lo, uint64_t rp, int* lo_nonzero) {
    pdl_enter();
    __shared__ float tile[64][65];
    const uint64_t c0 = (uint64_t)blockIdx.x * 64, r0 = (uint64_t)blockIdx.y * 64;
    const int tx = threadIdx.x % 64, ty = threadIdx.x / 64;  // 64 x 4
    for (int j = ty; j < 64; j += 4) {
        const uint64_t r = r0 + j, c = c0 + tx;
        tile[j][tx] = (r < r_count && c < c_count) ? src[r * c_count + c] : 0.0f;
    }
    __syncthreads();
    bool nz = false;
    for (int j = ty; j < 64; j += 4) {
        const uint64_t c = c0 + j, r = r0 + tx;
        if (c < c_count && r < rp) {
            float h, l;
            split_tf32(tile[tx][j], h, l);
            hi[c * rp + r] = h;
            lo[c * rp + r] = l;
            nz = nz || l != 0.0f;
        }
    }
    note_lo(lo_nonzero, nz);
}

// ---- the tensor-core GEMM ---------------------------------------------------------------------
struct TcParams {
    float* out;
    const float* addend;
    int addend_mode;
    uint64_t m, n, k;
    int tiles_m, tiles_n;
    int kb_per_split;  // k-blocks each CTA of a split handles
    int splits;        // CTAs per cluster (blockIdx.y), each over its own range of k
    int b_early;       // B is a stable prepared weight: its first loads may precede pdl_enter()
    int prefetch;      // prefetch tiles into the L2 one ring's depth ahead (one row of M tiles)
    int b_terms;       // 2; 1 when every B's lo term is zero (its values are exactly tf32): lo is
                       // neither loaded nor multiplied -- the products it would add are exact zeros
    int* error;        // device word set when a wait times out
    // Grouped projection: `groups` (1-3) weights multiply the same A side by side (tiles_n is
    // per weight); weight g writes outs[g] and, when rope_out[g] is set, also the rows of
    // outs[g] rotated by `rope` (interleaved pairs) into rope_out[g].
    int groups;
    float* outs[3];
    float* rope_out[3];
    RopeK rope;
};

// Split-k modes: kNoSplit; kSplitOwnRecv -- the receive slots have a region of their own (free
// from the start: no CTA waits for a peer's ring to drain before sending; costs ring depth);
// kSplitRingRecv -- the receive slots sit in the drained ring behind the staged tile (a cluster
// barrier after staging tells the senders every ring is drained; keeps the ring deep for long k).
constexpr int kNoSplit = 0, kSplitOwnRecv = 1, kSplitRingRecv = 2;

template <int BN, int NB, int STAGES, bool A_RAW, int SPLIT, bool B_RAW = false>
struct TcShape {
    static constexpr int kATile = BM * BK * 4;  // bytes of one A term tile
    static constexpr int kBTile = BN * BK * 4;  // bytes of one B term tile
    // B_RAW: TMA brings B's raw f32 [BK][BN] tile MN-major, as B lies in memory (boxes of
    // [32 k][32 n], 128-byte rows swizzled in 32-byte granules: the MMA's MN-major layout for
    // 32-bit operands), into the B hi slot; the converter warps split it element by element, hi
    // in place and lo into the lo slot at the same offsets -- no transpose.
    static constexpr int kStage = 2 * kATile + NB * 2 * kBTile;
    static constexpr int kTxBytes = (A_RAW ? 1 : 2) * kATile + (B_RAW ? NB : NB * 2) * kBTile;  // TMA bytes per stage
    static constexpr int kRing = STAGES * kStage;
    static constexpr int kLd = BN + 4;  // row stride (floats) of a staged tile and of the receive slots
    static_assert(NB * BM * kLd * 4 <= kRing, "the staged tile fits the drained ring");
    static constexpr int kBars = 512;
    // Split k: receive slots [NB][splits][band][kLd] for the other CTAs' partial rows of this
    // CTA's band.
    static constexpr int kStaged = NB * BM * kLd * 4;
    static constexpr int kRecvBytes = NB * (BM + kMaxSplits - 1) * kLd * 4;
    static_assert(SPLIT != kSplitRingRecv || kStaged + kRecvBytes <= kRing, "receive slots fit the drained ring");
    static constexpr int kRecv = SPLIT == kSplitOwnRecv ? kRecvBytes : 0;
    static constexpr int kSmem = kRing + kBars + kRecv + 1024 /* align */;
    // Tensor memory: the accumulators, then (raw A) each stage's A hi and lo terms, which the
    // converters store there and the MMAs read as their A operand.
    static constexpr int kTmemAcc = NB * BN;
    static constexpr int kTmemUsed = kTmemAcc + (A_RAW ? STAGES * 2 * BK : 0);
    static_assert(kTmemUsed <= 512, "accumulators and A terms fit the tensor memory");
    static constexpr uint32_t kTmemCols =
        kTmemUsed <= 32 ? 32 : kTmemUsed <= 64 ? 64 : kTmemUsed <= 128 ? 128 : kTmemUsed <= 256 ? 256 : 512;
    static constexpr int kThreads = (A_RAW || B_RAW) ? 320 : 192;
};

// The CTAs of one output tile form a cluster along blockIdx.y, each multiplying its own range
// of k.  After the main loop each CTA pushes the rows of its f32 accumulator into the shared
// memory of the CTA that owns their band; each CTA then sums its band's partials in
// cluster-rank order and writes the finished band with coalesced stores (bias / residual /
// SwiGLU applied).  One kernel, deterministic, and the partial sums never leave the chip.
template <int BN, int NB, int STAGES, bool A_RAW, int SPLIT, bool B_RAW>
__global__ void __launch_bounds__(TcShape<BN, NB, STAGES, A_RAW, SPLIT, B_RAW>::kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap map_a0, const __grid_constant__ CUtensorMap map_a1,
                   const __grid_constant__ CUtensorMap map_bhi, const __grid_constant__ CUtensorMap map_blo,
                   const __grid_constant__ CUtensorMap map_b2hi, const __grid_constant__ CUtensorMap map_b2lo,
                   const __grid_constant__ CUtensorMap map_b3hi, const __grid_constant__ CUtensorMap map_b3lo,
                   TcParams p) {
    using S = TcShape<BN, NB, STAGES, A_RAW, SPLIT, B_RAW>;
    constexpr bool kConvert = A_RAW || B_RAW;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* base_ptr = smem_raw + (base - raw);
    const uint32_t bar_base = base + S::kRing;
    uint64_t* bars = reinterpret_cast<uint64_t*>(base_ptr + S::kRing);
    // bars: [0, S) full (TMA), [S, 2S) empty (MMA done), [2S, 3S) converted, [3S] accumulator,
    // [3S + 1] split-k partials received
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(bars + 3 * STAGES + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 3 * STAGES + 3);
    auto full_bar = [&](int s) { return bar_base + 8u * s; };
    auto empty_bar = [&](int s) { return bar_base + 8u * (STAGES + s); };
    auto conv_bar = [&](int s) { return bar_base + 8u * (2 * STAGES + s); };
    const uint32_t accum_bar = bar_base + 8u * (3 * STAGES);
    const uint32_t recv_bar = bar_base + 8u * (3 * STAGES + 1);
    const uint32_t recv_base = SPLIT == kSplitOwnRecv ? bar_base + S::kBars : base + S::kStaged;
    // Split k: the CTAs of a tile's cluster each own one band of the tile's rows.
    const int splits = SPLIT ? p.splits : 1;
    const int rank = SPLIT ? (int)cooperative_groups::this_cluster().block_rank() : 0;
    const int band = (BM + splits - 1) / splits;
    const int r_begin = rank * band, r_end = min(BM, r_begin + band);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

    // Grouped rasterisation of the output tiles (blockIdx.x); blockIdx.y is the k split.
    const int tile = blockIdx.x;
    const int group_size = kGroupM * p.tiles_n * p.groups;
    const int group = tile / group_size;
    const int first_m = group * kGroupM;
    const int rows_in_group = min(p.tiles_m - first_m, kGroupM);
    const int tm = first_m + (tile % group_size) % rows_in_group;
    const int tn_all = (tile % group_size) / rows_in_group;
    const int wsel = tn_all / p.tiles_n;  // the weight of a grouped projection (0 otherwise)
    const int tn = tn_all - wsel * p.tiles_n;
    const int m0 = tm * BM, n0 = tn * BN;
    const CUtensorMap* map_whi = wsel == 0 ? &map_bhi : wsel == 1 ? &map_b2hi : &map_b3hi;
    const CUtensorMap* map_wlo = wsel == 0 ? &map_blo : wsel == 1 ? &map_b2lo : &map_b3lo;
    float* const outp = wsel == 0 ? p.outs[0] : wsel == 1 ? p.outs[1] : p.outs[2];
    float* const ropep = wsel == 0 ? p.rope_out[0] : wsel == 1 ? p.rope_out[1] : p.rope_out[2];
    const int num_kb_total = (int)((p.k + BK - 1) / BK);
    const int kb0 = blockIdx.y * p.kb_per_split;
    const int num_kb = max(0, min(num_kb_total, kb0 + p.kb_per_split) - kb0);

    // TMA loads of one stage (the producer's job): issue_b arms the stage's barrier for all
    // of the stage's bytes and loads B, issue_a loads A.
    auto issue_a = [&](int i) {
        const int s = i % STAGES;
        const uint32_t st = base + s * S::kStage;
        const int kx = (kb0 + i) * BK;
        tma_load_2d(st, &map_a0, full_bar(s), kx, m0);
        if (!A_RAW) tma_load_2d(st + S::kATile, &map_a1, full_bar(s), kx, m0);
    };
    auto issue_b = [&](int i) {
        const int s = i % STAGES;
        const uint32_t st = base + s * S::kStage;
        mbar_arrive_expect_tx(full_bar(s), S::kTxBytes - (B_RAW || p.b_terms == 2 ? 0 : NB * S::kBTile));
        const int kx = (kb0 + i) * BK;
        if (B_RAW) {
#pragma unroll
            for (int j = 0; j < BN / 32; j++) {  // [BK rows of k][32 columns] per box
                tma_load_2d(st + 2 * S::kATile + (uint32_t)(j * 32 * BK * 4), map_whi, full_bar(s), n0 + 32 * j, kx);
                if (NB == 2)  // the up weight into the second term's hi slot
                    tma_load_2d(st + 2 * S::kATile + 2 * S::kBTile + (uint32_t)(j * 32 * BK * 4), &map_b2hi, full_bar(s),
                                n0 + 32 * j, kx);
            }
            return;
        }
        tma_load_2d(st + 2 * S::kATile, map_whi, full_bar(s), kx, n0);
        if (p.b_terms == 2) tma_load_2d(st + 2 * S::kATile + S::kBTile, map_wlo, full_bar(s), kx, n0);
        if (NB == 2) {
            tma_load_2d(st + 2 * S::kATile + 2 * S::kBTile, &map_b2hi, full_bar(s), kx, n0);
            if (p.b_terms == 2) tma_load_2d(st + 2 * S::kATile + 3 * S::kBTile, &map_b2lo, full_bar(s), kx, n0);
        }
    };
    auto issue = [&](int i) {
        issue_b(i);
        issue_a(i);
    };
    // k-block i's tiles into the L2 one ring's depth ahead of their loads: the ring's loads
    // then wait on the L2, not on HBM, and twice the ring's bytes are on their way.  Only for
    // a single row of M tiles (B read once, latency-bound); with many rows it costs the L2
    // more than it saves (M = 8192: 1.21 -> 1.36 ms).
    auto prefetch = [&](int i) {
        if (!p.prefetch || i >= num_kb) return;
        const int kx = (kb0 + i) * BK;
        if (B_RAW) {
#pragma unroll
            for (int j = 0; j < BN / 32; j++) {
                tma_prefetch_2d(map_whi, n0 + 32 * j, kx);
                if (NB == 2) tma_prefetch_2d(&map_b2hi, n0 + 32 * j, kx);
            }
        } else {
            tma_prefetch_2d(map_whi, kx, n0);
            if (p.b_terms == 2) tma_prefetch_2d(map_wlo, kx, n0);
            if (NB == 2) {
                tma_prefetch_2d(&map_b2hi, kx, n0);
                if (p.b_terms == 2) tma_prefetch_2d(&map_b2lo, kx, n0);
            }
        }
        tma_prefetch_2d(&map_a0, kx, m0);
        if (!A_RAW) tma_prefetch_2d(&map_a1, kx, m0);
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
            mbar_init(conv_bar(s), kConvThreads / 32);
        }
        mbar_init(accum_bar, 1);
        if (SPLIT) mbar_init(recv_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
        // Arm the receive barrier for the other CTAs' partial rows of this CTA's band.
        if (SPLIT) mbar_arrive_expect_tx(recv_bar, (uint32_t)(NB * (splits - 1) * (r_end - r_begin) * S::kLd * 4));
        // A stable prepared weight is read by no earlier kernel's writes: its first stages
        // load while the previous kernel of the stream is still finishing.
        if (p.b_early)
            for (int i = 0; i < min(STAGES, num_kb); i++) issue_b(i);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32((const void*)tmem_slot), S::kTmemCols);
        tmem_relinquish();
    }
    // Cluster barrier, phase 1 (own receive region: arrive now, wait in the epilogue): every
    // CTA's receive barrier is initialised and armed before any CTA sends to it.
    if (SPLIT == kSplitOwnRecv) cluster_arrive();
    pdl_enter();
    // A residual addend is written by an earlier kernel: bring this CTA's band of it into the L2
    // now, so that the epilogue's loads of it do not wait on HBM.
    if (warp == 2 && p.addend_mode == 2) {
        constexpr int kLines = (BN * 4 + 127) / 128;  // 128-byte lines per band row
        for (int e = lane; e < (r_end - r_begin) * kLines; e += 32) {
            const uint64_t row = (uint64_t)m0 + r_begin + e / kLines, col = (uint64_t)n0 + (e % kLines) * 32;
            if (row < p.m && col < p.n)
                asm volatile("prefetch.global.L2 [%0];" ::"l"(p.addend + row * p.n + col) : "memory");
        }
    }
    if (threadIdx.x == 0) {
        // The first stages are free: start their loads before the set-up barrier so that the
        // memory latency overlaps the rest of the set-up.
        for (int i = 0; i < min(STAGES, num_kb); i++) {
            if (!p.b_early) issue_b(i);
            issue_a(i);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool acc_ready = false;  // warps 2-5: the accumulator is complete and valid

    if (warp == 0) {
        // ---- TMA producer --------------------------------------------------------------
        if (lane == 0) {
            // The next ring's worth of tiles goes to the L2 once the first stage has landed: issued
            // with the first stages, these prefetches would compete with them for HBM and delay
            // the start of the main loop.
            if (p.prefetch && num_kb > STAGES && mbar_wait(full_bar(0), 0))
                for (int i = STAGES; i < 2 * STAGES; i++) prefetch(i);
            for (int i = STAGES; i < num_kb; i++) {
                const int s = i % STAGES;
                const uint32_t phase = (uint32_t)(i / STAGES) & 1u;
                if (!mbar_wait(empty_bar(s), phase ^ 1u)) {
                    *abort_flag = 1;
                    atomicExch(p.error, 1);
                    break;
                }
                if (*abort_flag) break;
                issue(i);
                prefetch(i + STAGES);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---- MMA issuer ----------------------------------------------------------------
        if (lane == 0) {
            // raw B is MN-major (bit 16: B transposed)
            constexpr uint32_t idesc = idesc_tf32(BM, BN) | (B_RAW ? (1u << 16) : 0u);
            const bool two_b = B_RAW || p.b_terms == 2;
            bool ok = true;
            for (int i = 0; i < num_kb; i++) {
                const int s = i % STAGES;
                const uint32_t phase = (uint32_t)(i / STAGES) & 1u;
                if (!mbar_wait(full_bar(s), phase) || (kConvert && !mbar_wait(conv_bar(s), phase))) {
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
                const uint32_t ta = tmem + (uint32_t)(S::kTmemAcc + s * 2 * BK);  // raw A: hi, then lo
#pragma unroll
                for (int kk = 0; kk < BK / 8; kk++) {
                    const uint64_t koff = (uint64_t)((kk * 32) >> 4);  // 8 tf32 = 32 bytes
#pragma unroll
                    for (int z = 0; z < NB; z++) {
                        const uint32_t bt = st + 2 * S::kATile + z * 2 * S::kBTile;
                        // K-major terms advance 32 bytes per 8 k; MN-major raw B 8 rows (1 KB), its
                        // 32-column chunks 4 KB apart
                        const uint64_t bhi = B_RAW ? desc_mn_sw128_32b(bt + (uint32_t)(kk * 1024), 32 * BK * 4)
                                                   : desc_k_sw128(bt) + koff;
                        const uint64_t blo = B_RAW ? desc_mn_sw128_32b(bt + S::kBTile + (uint32_t)(kk * 1024), 32 * BK * 4)
                                                   : desc_k_sw128(bt + S::kBTile) + koff;
                        const uint32_t d = tmem + (uint32_t)(z * BN);
                        const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
                        if (A_RAW) {
                            const uint32_t ah = ta + (uint32_t)(kk * 8), al = ah + BK;
                            mma_tf32_ts(d, al, bhi, idesc, acc);
                            if (two_b) mma_tf32_ts(d, ah, blo, idesc, 1u);
                            mma_tf32_ts(d, ah, bhi, idesc, 1u);
                        } else {
                            mma_tf32(d, alo + koff, bhi, idesc, acc);
                            if (two_b) mma_tf32(d, ahi + koff, blo, idesc, 1u);
                            mma_tf32(d, ahi + koff, bhi, idesc, 1u);
                        }
                    }
                }
                tc_commit(empty_bar(s));  // frees the stage once these MMAs have read it
            }
            if (ok && num_kb > 0) tc_commit(accum_bar);
            else mbar_arrive(accum_bar);  // release the epilogue
        }
        __syncwarp();
    } else {
        // ---- warps 2..9 (raw operands): split each raw f32 A tile into hi (in place) + lo and
        //      each raw B tile into its K-major hi / lo terms, stage by stage ----------------
        if (kConvert) {
            const int t = threadIdx.x - 64;  // 0 .. kConvThreads - 1
            for (int i = 0; i < num_kb; i++) {
                const int s = i % STAGES;
                const uint32_t phase = (uint32_t)(i / STAGES) & 1u;
                if (!mbar_wait(full_bar(s), phase)) {
                    *abort_flag = 1;
                    atomicExch(p.error, 1);
                    // still arrive so that the MMA warp does not wait for us
                }
                const uint32_t st = base + s * S::kStage;
                if (A_RAW) {
                    // Row m of the raw A tile (this warp's lane quarter of the tensor memory), k half
                    // hp: its 16 values split into hi / lo and stored to the stage's A columns.  The
                    // MMAs that read these columns before have completed: the producer reloaded the
                    // stage only after they released it.
                    tc_fence_after();
                    const int q = warp % 4, hp = (warp - 2) / 4;
                    const int m = q * 32 + lane;
                    uint32_t hv[16], lv[16];
#pragma unroll
                    for (int c = 0; c < 4; c++) {
                        const int chunk = 4 * hp + c;  // 16-byte chunk of the 128-byte row, swizzled
                        float4 h, l;
                        split4_fast(lds4(st + (uint32_t)(m * 128 + ((chunk ^ (m & 7)) * 16))), h, l);
                        hv[4 * c] = __float_as_uint(h.x), hv[4 * c + 1] = __float_as_uint(h.y);
                        hv[4 * c + 2] = __float_as_uint(h.z), hv[4 * c + 3] = __float_as_uint(h.w);
                        lv[4 * c] = __float_as_uint(l.x), lv[4 * c + 1] = __float_as_uint(l.y);
                        lv[4 * c + 2] = __float_as_uint(l.z), lv[4 * c + 3] = __float_as_uint(l.w);
                    }
                    const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(S::kTmemAcc + s * 2 * BK + 16 * hp);
                    tmem_st16(ta, hv);
                    tmem_st16(ta + BK, lv);
                }
                if (B_RAW) {
                    // element by element: hi in place, lo at the same offset of the lo slot
#pragma unroll
                    for (int z = 0; z < NB; z++) {
                        const uint32_t b_hi = st + 2 * S::kATile + (uint32_t)(z * 2 * S::kBTile), b_lo = b_hi + S::kBTile;
#pragma unroll
                        for (int j = 0; j < S::kBTile / 16 / kConvThreads; j++) {
                            const uint32_t off = (uint32_t)(t + j * kConvThreads) * 16;
                            float4 h, l;
                            split4_fast(lds4(b_hi + off), h, l);
                            sts4(b_hi + off, h.x, h.y, h.z, h.w);
                            sts4(b_lo + off, l.x, l.y, l.z, l.w);
                        }
                    }
                }
                if (A_RAW) tc_wait_st();  // the A terms are in the tensor memory
                fence_proxy_async();      // make the generic-proxy writes visible to tcgen05.mma
                tc_fence_before();
                mbar_arrive_warp(conv_bar(s));
                if (__any_sync(0xffffffffu, *abort_flag)) break;
            }
        }
    }
    if (warp >= 2 && warp < 6) {
        // ---- warps 2..5: wait for the accumulator ------------------------------------------
        const bool waited = mbar_wait(accum_bar, 0);
        if (!waited) atomicExch(p.error, 1);
        // tcgen05.ld is warp-collective: the whole warp reads the accumulator or none of it.
        acc_ready = __all_sync(0xffffffffu, waited && !*abort_flag && num_kb > 0);
    }

    // ---- epilogue ------------------------------------------------------------------------
    // Warps 2-5 read their TMEM lane quarter and stage the tile in the drained ring
    // ([NB][BM][kLd]).  With split k, one thread then sends each band of the staged rows to the
    // CTA that owns it with one bulk copy into that CTA's receive slot for this split
    // (completing on the owner's receive barrier); each CTA sums its band's partials in split
    // order 0, 1, ... (deterministic) and writes the finished rows with coalesced stores, bias /
    // residual / SwiGLU applied.  The partial sums never leave the chip.
    if (warp >= 2 && warp < 6) {
        tc_fence_after();
        const int q = warp % 4;
        const int r = q * 32 + lane;  // this thread's row of the tile
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 32) {
#pragma unroll
            for (int z = 0; z < NB; z++) {
                float v[32];
                if (acc_ready) {
                    tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(z * BN + c0), v);
                    tc_wait_ld();
                } else {
#pragma unroll
                    for (int j = 0; j < 32; j++) v[j] = 0.0f;
                }
                const uint32_t dst = base + (uint32_t)(((z * BM + r) * S::kLd + c0) * 4);
#pragma unroll
                for (int j = 0; j < 32; j += 4) sts4(dst + 4 * j, v[j], v[j + 1], v[j + 2], v[j + 3]);
            }
        }
        if (SPLIT) fence_proxy_async();  // the staged rows are read by bulk copies next
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, S::kTmemCols);
    }
    if (SPLIT) {
        // Phase 1: every receive barrier of the cluster is armed (and, receiving in the ring,
        // every CTA has staged its tile: its ring is drained).
        if (SPLIT == kSplitRingRecv) cluster_arrive();
        cluster_wait();
        // Thread 64 + b sends band b (one issuing thread per destination).
        const int b = (int)threadIdx.x - 64;
        if (b >= 0 && b < splits && b != rank) {
            const int b_begin = b * band, b_rows = min(BM, b_begin + band) - b_begin;
#pragma unroll
            for (int z = 0; z < NB; z++) {
                const uint32_t src = base + (uint32_t)((z * BM + b_begin) * S::kLd * 4);
                const uint32_t dst = recv_base + (uint32_t)(((z * splits + rank) * band) * S::kLd * 4);
                bulk_copy_to_cluster(mapa(dst, (uint32_t)b), src, (uint32_t)(b_rows * S::kLd * 4),
                                     mapa(recv_bar, (uint32_t)b));
            }
        }
        if (!mbar_wait(recv_bar, 0)) atomicExch(p.error, 1);
        cluster_arrive();  // phase 2: every copy into this CTA has landed
    }
    // Address of row lr of this CTA's band, column c, term z, in split s's partial.
    auto part_at = [&](int z, int s, int lr, int c) -> uint32_t {
        return s == rank ? base + (uint32_t)(((z * BM + r_begin + lr) * S::kLd + c) * 4)
                         : recv_base + (uint32_t)((((z * splits + s) * band + lr) * S::kLd + c) * 4);
    };
    {
        constexpr int kVec = BN / 4;  // float4 per row
        const bool vec = (p.n % 4 == 0) && ((reinterpret_cast<uintptr_t>(outp) & 15) == 0) &&
                         (p.addend_mode == 0 || (reinterpret_cast<uintptr_t>(p.addend) & 15) == 0);
        for (int e = threadIdx.x; e < (r_end - r_begin) * kVec; e += blockDim.x) {
            const int lr = e / kVec, c4 = (e % kVec) * 4;
            const uint64_t row = (uint64_t)m0 + r_begin + lr, col = (uint64_t)n0 + c4;
            if (row >= p.m || col >= p.n) continue;
            const bool full4 = vec && col + 4 <= p.n;
            // The addend's global load goes out first, so that its latency overlaps the
            // shared-memory loads below.
            float4 add4 = make_float4(0.f, 0.f, 0.f, 0.f);
            if (full4 && p.addend_mode == 1) add4 = *reinterpret_cast<const float4*>(p.addend + col);
            else if (full4 && p.addend_mode == 2) add4 = *reinterpret_cast<const float4*>(p.addend + row * p.n + col);
            // the splits' partials in split order (deterministic), four loads in flight
            float4 acc[NB];
#pragma unroll
            for (int z = 0; z < NB; z++) {
                acc[z] = lds4(part_at(z, 0, lr, c4));
                for (int s0 = 1; s0 < splits; s0 += 4) {
                    float4 t[4];
#pragma unroll
                    for (int u = 0; u < 4; u++)
                        if (s0 + u < splits) t[u] = lds4(part_at(z, s0 + u, lr, c4));
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        if (s0 + u < splits) {
                            acc[z].x += t[u].x;
                            acc[z].y += t[u].y;
                            acc[z].z += t[u].z;
                            acc[z].w += t[u].w;
                        }
                    }
                }
            }
            float o[4] = {acc[0].x, acc[0].y, acc[0].z, acc[0].w};
            if (NB == 2) {
                const float u[4] = {acc[NB - 1].x, acc[NB - 1].y, acc[NB - 1].z, acc[NB - 1].w};
#pragma unroll
                for (int j = 0; j < 4; j++) o[j] = (o[j] * (1.0f / (1.0f + expf(-o[j])))) * u[j];
            }
            float* orow = outp + row * p.n;
            if (full4) {
                if (p.addend_mode != 0) o[0] += add4.x, o[1] += add4.y, o[2] += add4.z, o[3] += add4.w;
                *reinterpret_cast<float4*>(orow + col) = make_float4(o[0], o[1], o[2], o[3]);
                if (ropep) {
                    // RoPE of this float4 (two interleaved pairs of one head), the rope kernel's
                    // arithmetic on the same values.
                    const uint64_t ch = col % p.rope.head_width;
                    float4 y = make_float4(o[0], o[1], o[2], o[3]);
                    if (ch < p.rope.dimension) {
                        const float2 r0 = rope_cs(p.rope, row, ch >> 1), r1 = rope_cs(p.rope, row, (ch >> 1) + 1);
                        y.x = o[0] * r0.x - o[1] * r0.y;
                        y.y = o[0] * r0.y + o[1] * r0.x;
                        y.z = o[2] * r1.x - o[3] * r1.y;
                        y.w = o[2] * r1.y + o[3] * r1.x;
                    }
                    *reinterpret_cast<float4*>(ropep + row * p.n + col) = y;
                }
            } else {
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    if (col + j >= p.n) break;
                    float sum = o[j];
                    if (p.addend_mode == 1) sum += p.addend[col + j];
                    else if (p.addend_mode == 2) sum += p.addend[row * p.n + col + j];
                    orow[col + j] = sum;
                }
            }
        }
    }
    // Phase 2: every copy out of this CTA's shared memory has landed before the CTA exits.
    if (SPLIT) cluster_wait();
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

// K-major [rows, cols] f32 matrix (row stride ld elements), box [box_rows, 32] with 128-byte
// swizzle.
mg_status make_map(CUtensorMap* map, const float* ptr, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows) {
    auto fn = encode_fn();
    if (!fn) return fail(MG_DRIVER_FAILED, "the driver does not provide cuTensorMapEncodeTiled");
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld * sizeof(float)};
    cuuint32_t box[2] = {BK, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ptr), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(MG_DRIVER_FAILED, "encoding a TMA descriptor failed (CUresult %d)", (int)r);
    return MG_OK;
}

// B as it lies in memory, row-major [k, n] f32 (the MN-major operand): box [BK rows x 32 columns],
// 128-byte rows swizzled in 32-byte granules; rows and columns past the end read as zero.
mg_status make_raw_b_map(CUtensorMap* map, const float* b, uint64_t k, uint64_t n) {
    auto fn = encode_fn();
    if (!fn) return fail(MG_DRIVER_FAILED, "the driver does not provide cuTensorMapEncodeTiled");
    cuuint64_t dims[2] = {n, k};
    cuuint64_t strides[1] = {n * sizeof(float)};
    cuuint32_t box[2] = {32, BK};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(b), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
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
                        uint64_t kp, int* lo_nonzero = nullptr) {
    if (kmajor) {
        const int vec = k == kp && k % 4 == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0;
        enqueue(d, split_rows_kernel, grid_cap(d, vec ? rows * kp / 4 : rows * kp), 256, 0, src, k, rows, k, hi, lo,
                                                                                              kp, vec, lo_nonzero);
    } else {
        dim3 grid((unsigned)((rows + 63) / 64), (unsigned)((kp + 63) / 64));
        if (grid.y > 65535) return fail(MG_SHAPE_UNSUPPORTED, "matmul inner dimension %llu is too large", (unsigned long long)k);
        enqueue(d, split_transpose_kernel, grid, 256, 0, src, k, rows, hi, lo, kp, lo_nonzero);
    }
    return launched(d, "operand split kernel launch");
}

template <int BN, int NB, int STAGES, bool A_RAW, int SPLIT, bool B_RAW = false>
mg_status launch_tc(Device* d, TcParams p, const CUtensorMap* maps) {
    using S = TcShape<BN, NB, STAGES, A_RAW, SPLIT, B_RAW>;
    static_assert(S::kSmem <= 227 * 1024, "shared memory budget");
    auto kernel = gemm_tc_kernel<BN, NB, STAGES, A_RAW, SPLIT, B_RAW>;
    static bool configured[64] = {false};
    if (!configured[d->ordinal & 63]) {
        MG_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmem),
                "configuring the tensor-core matmul");
        if (SPLIT)
            MG_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1),
                    "allowing the tensor-core matmul clusters of up to 16");
        configured[d->ordinal & 63] = true;
    }
    const uint64_t tiles = (uint64_t)p.tiles_m * p.tiles_n * p.groups;
    if (tiles > 0x7FFFFFFFull) return fail(MG_SHAPE_UNSUPPORTED, "matmul has too many output tiles");
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(S::kThreads, 1, 1);
    cfg.dynamicSmemBytes = S::kSmem;
    cfg.stream = d->stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    if (SPLIT) {
        // Keep the clusters to one wave: fewer splits when the GPCs cannot hold `tiles`
        // clusters of this size at once (queried once per cluster size).
        static int max_clusters[kMaxSplits + 1] = {0};
        const int num_kb = (int)((p.k + BK - 1) / BK);
        while (p.splits > 2) {
            int& mc = max_clusters[p.splits];
            if (mc == 0) {
                attr[0].val.clusterDim.y = (unsigned)p.splits;
                cfg.gridDim = dim3((unsigned)tiles, (unsigned)p.splits, 1);
                cfg.numAttrs = 1;
                if (cudaOccupancyMaxActiveClusters(&mc, kernel, &cfg) != cudaSuccess || mc <= 0) {
                    (void)cudaGetLastError();
                    mc = 1 << 30;  // unknown: assume it fits
                }
            }
            if ((uint64_t)mc >= tiles) break;
            p.splits--;
            p.kb_per_split = (num_kb + p.splits - 1) / p.splits;
            p.splits = (num_kb + p.kb_per_split - 1) / p.kb_per_split;
        }
    }
    attr[0].val.clusterDim.y = (unsigned)p.splits;  // the k splits of one tile share a cluster
    cfg.gridDim = dim3((unsigned)tiles, (unsigned)p.splits, 1);
    cfg.numAttrs = d->pdl ? 2 : 1;
    MG_CUDA(cudaLaunchKernelEx(&cfg, kernel, maps[0], maps[1], maps[2], maps[3], maps[4], maps[5], maps[6], maps[7], p),
            "tensor-core matmul launch");
    return launched(d, "tensor-core matmul launch");
}

// Ring depth per tile width: as deep as the shared memory allows.  Split k with few k-blocks
// per CTA (the decoder layer's GEMMs) takes its own receive region and a shallower ring, so no
// CTA waits for its peers before sending; with many k-blocks per CTA the ring depth matters more
// and the partials are received in the drained ring.
template <int NB, bool A_RAW>
mg_status launch_bn(Device* d, int bn, const TcParams& p, const CUtensorMap* maps) {
    const int mode = p.splits <= 1 ? kNoSplit : p.kb_per_split < 8 ? kSplitOwnRecv : kSplitRingRecv;
    if constexpr (NB == 2) {
        if (bn == 128 && mode == kNoSplit) return launch_tc<128, NB, 2, A_RAW, kNoSplit>(d, p, maps);
        if (bn == 64) {
            if (mode == kNoSplit) return launch_tc<64, NB, 3, A_RAW, kNoSplit>(d, p, maps);
            if (mode == kSplitOwnRecv) return launch_tc<64, NB, 2, A_RAW, kSplitOwnRecv>(d, p, maps);
            return launch_tc<64, NB, 3, A_RAW, kSplitRingRecv>(d, p, maps);
        }
        if (bn == 32) {
            if (mode == kNoSplit) return launch_tc<32, NB, 4, A_RAW, kNoSplit>(d, p, maps);
            if (mode == kSplitOwnRecv) return launch_tc<32, NB, 3, A_RAW, kSplitOwnRecv>(d, p, maps);
            return launch_tc<32, NB, 4, A_RAW, kSplitRingRecv>(d, p, maps);
        }
        return fail(MG_EXECUTION_FAILED, "gated matmul tile width %d with split k", bn);
    } else {
        if (bn == 128) {
            if (mode == kNoSplit) return launch_tc<128, NB, 3, A_RAW, kNoSplit>(d, p, maps);
            if (mode == kSplitOwnRecv) return launch_tc<128, NB, 2, A_RAW, kSplitOwnRecv>(d, p, maps);
            return launch_tc<128, NB, 3, A_RAW, kSplitRingRecv>(d, p, maps);
        }
        if (bn == 64) {
            if (mode == kNoSplit) return launch_tc<64, NB, 4, A_RAW, kNoSplit>(d, p, maps);
            if (mode == kSplitOwnRecv) return launch_tc<64, NB, 3, A_RAW, kSplitOwnRecv>(d, p, maps);
            return launch_tc<64, NB, 4, A_RAW, kSplitRingRecv>(d, p, maps);
        }
        if (mode == kNoSplit) return launch_tc<32, NB, 5, A_RAW, kNoSplit>(d, p, maps);
        if (mode == kSplitOwnRecv) return launch_tc<32, NB, 4, A_RAW, kSplitOwnRecv>(d, p, maps);
        return launch_tc<32, NB, 5, A_RAW, kSplitRingRecv>(d, p, maps);
    }
}

// Raw B: its raw tile lands in the B hi slot, so the stage has the size of the terms' stage and
// the ring the same depth.
template <bool A_RAW>
mg_status launch_bn_raw_b(Device* d, int bn, const TcParams& p, const CUtensorMap* maps) {
    const int mode = p.splits <= 1 ? kNoSplit : p.kb_per_split < 8 ? kSplitOwnRecv : kSplitRingRecv;
    if (bn == 128) {
        if (mode == kNoSplit) return launch_tc<128, 1, 3, A_RAW, kNoSplit, true>(d, p, maps);
        if (mode == kSplitOwnRecv) return launch_tc<128, 1, 2, A_RAW, kSplitOwnRecv, true>(d, p, maps);
        return launch_tc<128, 1, 3, A_RAW, kSplitRingRecv, true>(d, p, maps);
    }
    if (bn == 64) {
        if (mode == kNoSplit) return launch_tc<64, 1, 4, A_RAW, kNoSplit, true>(d, p, maps);
        if (mode == kSplitOwnRecv) return launch_tc<64, 1, 3, A_RAW, kSplitOwnRecv, true>(d, p, maps);
        return launch_tc<64, 1, 4, A_RAW, kSplitRingRecv, true>(d, p, maps);
    }
    if (mode == kNoSplit) return launch_tc<32, 1, 5, A_RAW, kNoSplit, true>(d, p, maps);
    if (mode == kSplitOwnRecv) return launch_tc<32, 1, 4, A_RAW, kSplitOwnRecv, true>(d, p, maps);
    return launch_tc<32, 1, 5, A_RAW, kSplitRingRecv, true>(d, p, maps);
}

template <bool A_RAW>
mg_status launch_bn_raw_b2(Device* d, int bn, const TcParams& p, const CUtensorMap* maps) {
    const int mode = p.splits <= 1 ? kNoSplit : p.kb_per_split < 8 ? kSplitOwnRecv : kSplitRingRecv;
    if (bn == 128 && mode == kNoSplit) return launch_tc<128, 2, 2, A_RAW, kNoSplit, true>(d, p, maps);
    if (bn == 64) {
        if (mode == kNoSplit) return launch_tc<64, 2, 3, A_RAW, kNoSplit, true>(d, p, maps);
        if (mode == kSplitOwnRecv) return launch_tc<64, 2, 2, A_RAW, kSplitOwnRecv, true>(d, p, maps);
        return launch_tc<64, 2, 3, A_RAW, kSplitRingRecv, true>(d, p, maps);
    }
    if (bn == 32) {
        if (mode == kNoSplit) return launch_tc<32, 2, 4, A_RAW, kNoSplit, true>(d, p, maps);
        if (mode == kSplitOwnRecv) return launch_tc<32, 2, 3, A_RAW, kSplitOwnRecv, true>(d, p, maps);
        return launch_tc<32, 2, 4, A_RAW, kSplitRingRecv, true>(d, p, maps);
    }
    return fail(MG_EXECUTION_FAILED, "gated matmul tile width %d with split k", bn);
}

// k splits per tile at most (MAGNETAR_CUDA_GEMM_MAX_SPLITS, 2..16): the CTAs of one cluster,
// portable up to 8; 16 where the GPU holds such clusters (launch_tc checks).  Measured with 16
// against 8: 128 x 1376 x 512 (the decoder layer's down projection) 9.3 against 9.9 us; the other
// layer shapes and M = 128 x 4096 x 4096 unchanged.
int max_splits() {
    static int v = [] {
        const char* e = getenv("MAGNETAR_CUDA_GEMM_MAX_SPLITS");
        const int x = e ? atoi(e) : 16;
        return x < 2 ? 2 : x > kMaxSplits ? kMaxSplits : x;
    }();
    return v;
}

bool tensor_cores_enabled() {
    static int enabled = -1;
    if (enabled < 0) {
        const char* v = getenv("MAGNETAR_CUDA_TENSOR_CORES");
        enabled = (v && strcmp(v, "0") == 0) ? 0 : 1;
    }
    return enabled == 1;
}

// Output tile width: 128, except that a single row of tiles narrow enough to need deep k
// splits (128 x 512 x 512 in the decoder layer: 8 splits of 4 tiles) uses 64-wide tiles -- the
// same MMA work over twice the CTAs with half the split-k exchange per CTA (measured per call:
// 4.7 vs 6.5 us at k = 512, 8.5 vs 14.1 us at k = 1376; at n = 4096, 128 wide stays faster).
int pick_bn(const Device* d, uint64_t m, uint64_t n) {
    if (n <= 32) return 32;
    if (n <= 64) return 64;
    if (m <= 128 && ((n + 127) / 128) * 8 <= (uint64_t)d->sm_count) return 64;
    return 128;
}

}  // namespace

namespace k {

// One launch for `count` (1-3) matmuls that share A and their shape: a grouped projection
// (the decoder layer's q, k and v), each optionally also written rotated by `rope`
// (rope_outs[i], or null).  count > 1 or a rope needs plain matmuls: no gate, no addend, no
// transposes, f32 rows with 16-byte alignment; the caller checks (gemm_group_eligible).
mg_status gemm_tc_group(Device* d, const GemmArgs* gs, int count, const RopeK* rope, float* const* rope_outs) {
    const GemmArgs& g = gs[0];
    const uint64_t kp = gemm_kp(g.k);  // TMA row strides are multiples of 16 bytes
    const int nb = g.gated ? 2 : 1;
    // A: raw through TMA (split inside the kernel) when it is K-major with 16-byte rows and
    // small -- this saves a launch, but the in-kernel split costs shared-memory bandwidth in
    // the main loop, so large A (M = 2048: 0.48 vs 0.45 ms measured) takes a split pass.
    const bool a_raw = !g.transpose_a && g.k % 4 == 0 && (reinterpret_cast<uintptr_t>(g.a) & 15) == 0 && g.m <= 512;
    const float* ahi = g.a;
    const float* alo = nullptr;
    if (!a_raw) {
        float* a_split = nullptr;
        MG_TRY(scratch(d, 1, 2 * g.m * kp * sizeof(float), (void**)&a_split));
        MG_TRY(split_operand(d, g.a, g.m, g.k, !g.transpose_a, a_split, a_split + g.m * kp, kp));
        ahi = a_split;
        alo = a_split + g.m * kp;
    }
    // B raw (split in the kernel, no separate pass over B): with one row of tiles (M <= 128), for
    // a B that has no prepared form.  Its tiles arrive MN-major as B lies, the MMA reads them so,
    // and the converters split each element in place (hi) and beside it (lo).  Measured at
    // K = N = 4096, M = 128: 34.5 us against 44.7 us with a split pass.
    // A weight's prepared hi / lo form costs twice its f32 bytes per read.  Raw weights halve
    // that at the same speed for k <= 2048 (the decoder layer's projections: 55.35 vs 55.37 us per
    // step, the gated node 11.8 vs 12.0 us), while at K = N = 4096 the prepared form is faster
    // (32.8 vs 34.4 us: the main loop is bound by the 3xTF32 MMAs, and the converters' extra pass
    // costs more than the halved weight traffic saves).  So weights are read raw up to k = 2048;
    // MAGNETAR_CUDA_GEMM_RAW_WEIGHTS=0 / 1 reads them prepared / raw at every k.
    auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    static const int raw_weights_env = [] {
        const char* e = getenv("MAGNETAR_CUDA_GEMM_RAW_WEIGHTS");
        return e && *e ? (atoi(e) != 0 ? 1 : 0) : -1;
    }();
    const bool raw_weights = raw_weights_env > 0 || (raw_weights_env < 0 && g.k <= 2048);
    // The same for a gated matmul (gate and up both raw) and a grouped projection (every weight
    // raw); a weight whose prepared lo term is zero keeps its one-term prepared form.
    auto raw_ok = [&](const float* b, const float* prep, int one_term) {
        return b && al16(b) && (prep == nullptr || (raw_weights && !one_term));
    };
    bool b_raw = !g.transpose_b && g.n % 4 == 0 && !g.packed[0] && !g.packed[1] && g.m <= 128;
    if (nb == 2) {
        b_raw = b_raw && raw_ok(g.b, g.b_prep[0], g.b_one_term[0]) && raw_ok(g.b2, g.b_prep[1], g.b_one_term[1]);
    } else {
        for (int w = 0; w < count; w++) b_raw = b_raw && raw_ok(gs[w].b, gs[w].b_prep[0], gs[w].b_one_term[0]);
    }
    // B terms: [term or weight] -> hi, lo ([n, kp] each)
    const int nw = nb == 2 ? 2 : count;
    const float* bhi[3];
    const float* blo[3];
    int need_split = 0;
    for (int w = 0; w < nw && !b_raw; w++) need_split += (nb == 2 ? g.b_prep[w] : gs[w].b_prep[0]) == nullptr;
    float* b_split = nullptr;
    if (need_split) MG_TRY(scratch(d, 2, (size_t)nw * 2 * g.n * kp * sizeof(float), (void**)&b_split));
    bool stable = true;
    for (int w = 0; w < nw && !b_raw; w++) {
        const float* prep = nb == 2 ? g.b_prep[w] : gs[w].b_prep[0];
        stable = stable && prep && (nb == 2 ? g.b_stable : gs[w].b_stable);
        if (prep) {
            bhi[w] = prep;
            blo[w] = prep + g.n * kp;
        } else {
            float* hi = b_split + (size_t)w * 2 * g.n * kp;
            float* lo = hi + g.n * kp;
            const float* src = nb == 2 ? (w ? g.b2 : g.b) : gs[w].b;
            MG_TRY(split_operand(d, src, g.n, g.k, g.transpose_b != 0, hi, lo, kp));
            bhi[w] = hi;
            blo[w] = lo;
        }
    }
    int bn = pick_bn(d, g.m, g.n * (uint64_t)count);
    TcParams p;
    p.out = g.out;
    p.addend = g.addend;
    p.addend_mode = g.addend_mode;
    p.m = g.m;
    p.n = g.n;
    p.k = g.k;
    p.error = d->flags + 2;
    // raw B may load early when it is a weight (nothing earlier in the stream writes it)
    bool raw_stable = true;
    for (int w = 0; w < (nb == 2 ? 1 : count); w++) raw_stable = raw_stable && gs[w].b_stable != 0;
    p.b_early = (b_raw ? raw_stable : stable) ? 1 : 0;
    p.prefetch = g.m <= 128 ? 1 : 0;
    // One B term when every weight read is a prepared form whose lo term is all zero.
    bool one_term = !b_raw;
    for (int w = 0; w < nw && one_term; w++)
        one_term = (nb == 2 ? g.b_prep[w] && g.b_one_term[w] : gs[w].b_prep[0] && gs[w].b_one_term[0]) != 0;
    p.b_terms = one_term ? 1 : 2;
    p.groups = count;
    for (int i = 0; i < 3; i++) {
        p.outs[i] = i < count ? gs[i].out : nullptr;
        p.rope_out[i] = i < count && rope_outs ? rope_outs[i] : nullptr;
    }
    if (rope) p.rope = *rope;
    else memset(&p.rope, 0, sizeof p.rope);
    // Split k when the output grid leaves SMs idle: as many splits as fit in one wave, at
    // least 2 k-blocks each.  A gated split-k tile is at most 64 wide (its receive slots
    // share the shared memory with the ring).
    const int num_kb = (int)((g.k + BK - 1) / BK);
    auto plan_splits = [&](int width) {
        p.tiles_m = (int)((g.m + BM - 1) / BM);
        p.tiles_n = (int)((g.n + width - 1) / width);
        const uint64_t tiles = (uint64_t)p.tiles_m * p.tiles_n * count;
        int splits = 1;
        if (tiles * 2 <= (uint64_t)d->sm_count && num_kb >= 4) {
            splits = (int)((uint64_t)d->sm_count / tiles);
            if (splits > num_kb / 2) splits = num_kb / 2;
            if (splits > max_splits()) splits = max_splits();
            if (splits < 1) splits = 1;
        }
        p.kb_per_split = (num_kb + splits - 1) / splits;
        p.splits = (num_kb + p.kb_per_split - 1) / p.kb_per_split;
    };
    plan_splits(bn);
    if (nb == 2 && bn == 128 && p.splits > 1) {
        bn = 64;
        plan_splits(bn);
    }
    CUtensorMap maps[8];
    if (a_raw) {
        MG_TRY(make_map(&maps[0], ahi, g.m, g.k, g.k, BM));
        maps[1] = maps[0];
    } else {
        MG_TRY(make_map(&maps[0], ahi, g.m, kp, kp, BM));
        MG_TRY(make_map(&maps[1], alo, g.m, kp, kp, BM));
    }
    for (int w = 0; w < 3; w++) {
        if (b_raw) {
            // weight w's raw map in its hi slot (the lo slot unused)
            if (w < nw) MG_TRY(make_raw_b_map(&maps[2 + 2 * w], nb == 2 ? (w ? g.b2 : g.b) : gs[w].b, g.k, g.n));
            else maps[2 + 2 * w] = maps[2];
            maps[3 + 2 * w] = maps[2 + 2 * w];
        } else if (w < nw) {
            MG_TRY(make_map(&maps[2 + 2 * w], bhi[w], g.n, kp, kp, bn));
            MG_TRY(make_map(&maps[3 + 2 * w], blo[w], g.n, kp, kp, bn));
        } else {
            maps[2 + 2 * w] = maps[2];
            maps[3 + 2 * w] = maps[3];
        }
    }
    if (b_raw && nb == 2) return a_raw ? launch_bn_raw_b2<true>(d, bn, p, maps) : launch_bn_raw_b2<false>(d, bn, p, maps);
    if (b_raw) return a_raw ? launch_bn_raw_b<true>(d, bn, p, maps) : launch_bn_raw_b<false>(d, bn, p, maps);
    mg_status s;
    if (nb == 2) s = a_raw ? launch_bn<2, true>(d, bn, p, maps) : launch_bn<2, false>(d, bn, p, maps);
    else s = a_raw ? launch_bn<1, true>(d, bn, p, maps) : launch_bn<1, false>(d, bn, p, maps);
    MG_TRY(s);
    return MG_OK;
}

mg_status gemm_tc(Device* d, const GemmArgs& g) { return gemm_tc_group(d, &g, 1, nullptr, nullptr); }

bool gemm_group_eligible(const GemmArgs* gs, int count, const RopeArgs* rope, float* const* rope_outs) {
    if (count < 1 || count > 3) return false;
    auto al = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    const GemmArgs& g = gs[0];
    if (!gemm_uses_tensor_cores(g.m, g.n, g.k, 0, g.b) || g.n % 4 != 0) return false;
    for (int i = 0; i < count; i++) {
        const GemmArgs& x = gs[i];
        if (x.gated || x.addend_mode != 0 || x.transpose_a || x.transpose_b || x.a != g.a || x.m != g.m ||
            x.n != g.n || x.k != g.k || !al(x.out))
            return false;
        if (rope_outs && rope_outs[i] && !al(rope_outs[i])) return false;
    }
    if (rope) {  // interleaved pairs whose float4 groups never straddle a head or the rotary part
        const uint64_t hw = rope->cols / rope->head_count;
        if (rope->half_split || rope->cols != g.n || rope->rows != g.m || hw % 4 != 0 || rope->dimension % 4 != 0)
            return false;
    }
    return true;
}

mg_status gemm_group(Device* d, const GemmArgs* gs, int count, const RopeArgs* rope, float* const* rope_outs) {
    if (!gemm_group_eligible(gs, count, rope, rope_outs))
        return fail(MG_EXECUTION_FAILED, "matmul group is not eligible for one launch");
    RopeK rk;
    memset(&rk, 0, sizeof rk);
    if (rope) {
        rk.rows = rope->rows;
        rk.cols = rope->cols;
        rk.half = rope->half;
        rk.dimension = rope->dimension;
        rk.position_offset = rope->position_offset;
        rk.step = rope->step;
        rk.head_count = rope->head_count;
        rk.head_width = rope->cols / rope->head_count;
        rk.rotated_pairs = rope->rotated_pairs;
        rk.base = rope->base;
        rk.scale = rope->scale;
        rk.banded_factor = rope->banded_factor;
        rk.low_freq_factor = rope->low_freq_factor;
        rk.high_freq_factor = rope->high_freq_factor;
        rk.original_context_length = rope->original_context_length;
        rk.yarn_factor = rope->yarn_factor;
        rk.yarn_low = rope->yarn_low;
        rk.yarn_high = rope->yarn_high;
        rk.amplitude = rope->amplitude;
        rk.half_split = 0;
        rk.vec = 1;
    }
    return gemm_tc_group(d, gs, count, rope ? &rk : nullptr, rope_outs);
}

bool gemm_uses_tensor_cores(uint64_t m, uint64_t n, uint64_t k, int transpose_b, const float* b) {
    if (m == 0 || n == 0 || k == 0) return false;
    GemmArgs probe{};
    probe.m = m;
    probe.n = n;
    probe.k = k;
    probe.transpose_b = transpose_b;
    probe.b = b;
    if (gemv_eligible(probe)) return false;
    return tensor_cores_enabled() && m > 16;
}

mg_status gemm_prepare_b(Device* d, const float* b, uint64_t k, uint64_t n, int transposed, float* dst,
                         int* lo_nonzero) {
    const uint64_t kp = gemm_kp(k);
    return split_operand(d, b, n, k, transposed != 0, dst, dst + n * kp, kp, lo_nonzero);
}

mg_status gemm(Device* d, const GemmArgs& g) {
    if (g.m == 0 || g.n == 0) return MG_OK;
    if (g.packed[0] || g.packed[1]) return q8_matmul(d, g);
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
