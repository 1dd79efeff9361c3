// Fused causal / windowed / GQA attention on the 5th-generation tensor cores.
//
// The reference's tensor-core prefill (`attention_tcp{,128}_kernel`, src/tensor_kernels.cu:
// 755-1022) splits each f32 operand into bfloat16 hi + lo terms and forms
// hi*hi + hi*lo + lo*hi for both S = Q K^T and O = P V.  This kernel keeps that precision model
// on tcgen05:
//   * a split pass writes Q and K as bf16 hi/lo (same layout) and V as bf16 hi/lo transposed
//     per kv head ([kv_heads * D, keys]), so every MMA operand is K-major;
//   * a CTA serves 128 queries of one head.  Warp 0 loads Q once and 64-key tiles of K and
//     V^T with TMA; warp 1 issues the MMAs (S into TMEM columns [0, 64), P.V into [128, 128+D));
//     warps 4-7 -- one TMEM lane quarter each, one query row per thread -- read S, apply the
//     masks, run the online softmax, write P (normalised by the running sum) as bf16 hi/lo in
//     the 128-byte-swizzled layout the MMA reads, and fold each tile's P.V into a register
//     copy of the output.
// The output is kept as a weighted MEAN of V rows at every step (O <- O * l_old*a/l_new +
// (P/l_new) V), so it never exceeds the largest |v| -- the reference's overflow-safety
// invariant for large finite V (src/tests_conformance.rs:884-914).  A query with no admitted
// key outputs zeros.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>

#include <cstdlib>
#include <mutex>
#include <type_traits>

#include "internal.h"
#include "sm100.cuh"

namespace mg {
namespace {

using namespace sm100;

constexpr int AQ = 128;   // queries per CTA (MMA M)
constexpr int AKV = 64;   // keys per iteration (one 128-byte swizzle row of bf16)
constexpr int kAttnTcThreads = 384;  // 12 warps: producer, MMA, 2 idle, 8 softmax

// ---- split pass -----------------------------------------------------------------------------
__device__ __forceinline__ void split_bf16(float x, uint16_t& hi, uint16_t& lo) {
    __nv_bfloat16 h = __float2bfloat16_rn(x);
    float hf = __bfloat162float(h);
    if (isinf(hf) && !isinf(x)) {  // rounding overflowed a finite value: truncate instead
        const uint16_t t = (uint16_t)(__float_as_uint(x) >> 16);
        h = __ushort_as_bfloat16(t);
        hf = __bfloat162float(h);
    }
    hi = __bfloat16_as_ushort(h);
    lo = __bfloat16_as_ushort(__float2bfloat16_rn(x - hf));
}

__device__ __forceinline__ uint32_t pack_bf16(uint16_t a, uint16_t b) { return a | ((uint32_t)b << 16); }

// [rows, cols] f32 -> bf16 hi / lo in the same layout; four 16-byte loads in flight per thread.
// `clear` (optional): a word zeroed by the first thread (the V pass's max |v| of this call).
__global__ void __launch_bounds__(256) split_bf16_rows_kernel(const float* __restrict__ src, uint16_t* __restrict__ hi,
                                                              uint16_t* __restrict__ lo, uint64_t n, unsigned* clear) {
    pdl_enter();
    if (clear && blockIdx.x == 0 && threadIdx.x == 0) *clear = 0u;
    const uint64_t n4 = n / 4, stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i0 = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < n4; i0 += 4 * stride) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const uint64_t i = i0 + u * stride;
            if (i < n4) v[u] = reinterpret_cast<const float4*>(src)[i];
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const uint64_t i = i0 + u * stride;
            if (i >= n4) break;
            uint16_t h[4], l[4];
            split_bf16(v[u].x, h[0], l[0]);
            split_bf16(v[u].y, h[1], l[1]);
            split_bf16(v[u].z, h[2], l[2]);
            split_bf16(v[u].w, h[3], l[3]);
            reinterpret_cast<uint2*>(hi)[i] = make_uint2(pack_bf16(h[0], h[1]), pack_bf16(h[2], h[3]));
            reinterpret_cast<uint2*>(lo)[i] = make_uint2(pack_bf16(l[0], l[1]), pack_bf16(l[2], l[3]));
        }
    }
}

// v [keys, width] f32 -> hi / lo [width, keys_p] bf16 (dst[c][r] = v[r][c]), zero past keys.
// One CTA per 64 x 64 tile: 16-byte loads along v's rows, and each output row segment (64
// keys, 128 bytes) written by eight lanes with 16-byte stores.  The bits of max |v| (NaN above
// every number) go to *vmax.
__global__ void __launch_bounds__(256) split_bf16_transpose_kernel(const float* __restrict__ v, uint64_t keys,
                                                                   uint64_t width, uint16_t* __restrict__ hi,
                                                                   uint16_t* __restrict__ lo, uint64_t keys_p,
                                                                   unsigned* vmax) {
    pdl_enter();
    __shared__ float tile[64][65];  // [key][column]
    unsigned amax = 0u;
    const uint64_t c0 = (uint64_t)blockIdx.x * 64, r0 = (uint64_t)blockIdx.y * 64;
    const bool vec = width % 4 == 0 && c0 + 64 <= width;
    for (int e = threadIdx.x; e < 64 * 16; e += 256) {
        const int r = e / 16, q = e % 16;
        const uint64_t row = r0 + r, col = c0 + 4 * q;
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        if (row < keys) {
            if (vec) {
                x = *reinterpret_cast<const float4*>(v + row * width + col);
            } else {
                const float* p = v + row * width;
                if (col < width) x.x = p[col];
                if (col + 1 < width) x.y = p[col + 1];
                if (col + 2 < width) x.z = p[col + 2];
                if (col + 3 < width) x.w = p[col + 3];
            }
        }
        tile[r][4 * q] = x.x;
        tile[r][4 * q + 1] = x.y;
        tile[r][4 * q + 2] = x.z;
        tile[r][4 * q + 3] = x.w;
        amax = max(max(amax, max(__float_as_uint(x.x) & 0x7FFFFFFFu, __float_as_uint(x.y) & 0x7FFFFFFFu)),
                   max(__float_as_uint(x.z) & 0x7FFFFFFFu, __float_as_uint(x.w) & 0x7FFFFFFFu));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = max(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((threadIdx.x & 31) == 0 && amax) atomicMax(vmax, amax);
    __syncthreads();
    const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
    for (int cc = warp * 4 + lane / 8; cc < 64; cc += 32) {  // 4 columns per warp and turn
        const uint64_t col = c0 + cc;
        const int k8 = (lane % 8) * 8;  // this lane's 8 keys of the column
        const uint64_t key = r0 + k8;
        if (col >= width || key >= keys_p) continue;
        uint16_t h[8], l[8];
#pragma unroll
        for (int j = 0; j < 8; j++) split_bf16(tile[k8 + j][cc], h[j], l[j]);
        uint16_t* dh = hi + col * keys_p + key;
        uint16_t* dl = lo + col * keys_p + key;
        if (key + 8 <= keys_p && (keys_p % 8) == 0) {
            *reinterpret_cast<uint4*>(dh) = make_uint4(pack_bf16(h[0], h[1]), pack_bf16(h[2], h[3]), pack_bf16(h[4], h[5]), pack_bf16(h[6], h[7]));
            *reinterpret_cast<uint4*>(dl) = make_uint4(pack_bf16(l[0], l[1]), pack_bf16(l[2], l[3]), pack_bf16(l[4], l[5]), pack_bf16(l[6], l[7]));
        } else {
            for (int j = 0; j < 8 && key + j < keys_p; j++) {
                dh[j] = h[j];
                dl[j] = l[j];
            }
        }
    }
}

// ---- the attention kernel -----------------------------------------------------------------------
struct AttnTcParams {
    float* out;
    uint64_t seq_len, kv_seq_len, group, out_dim;
    int causal;
    int64_t window;  // -1: none
    uint64_t qpos0;  // position of query 0
    float scale;
    int q_tiles;
    int* error;
};

template <int D>
struct AttnShape {
    static constexpr int kQAtom = AQ * 128;          // [128 rows][64 bf16]
    static constexpr int kQ = (D / 64) * kQAtom;     // one term of the Q tile
    static constexpr int kKAtom = AKV * 128;         // [64 keys][64 bf16]
    static constexpr int kK = (D / 64) * kKAtom;     // one term of a K tile
    static constexpr int kV = D * 128;               // one term of a V^T tile: [D][64 keys]
    static constexpr int kP = AQ * 128;              // one term of P: [128][64 keys]
    // K is double-buffered (slot b: hi at kOffK + 2 * b * kK, lo right after): the next tile's K
    // loads while this tile's scores are computed.
    static constexpr int kOffQ = 0, kOffK = 2 * kQ, kOffV = kOffK + 4 * kK, kOffP = kOffV + 2 * kV;
    static constexpr int kBytes = kOffP + 2 * kP;
    static constexpr int kSmem = kBytes + 1024 + 256;
    static constexpr uint32_t kTmemCols = 256;       // S: [0, 64) and [64, 128), P.V: [128, 128 + D)
    static constexpr uint32_t kColPV = 128;
    static constexpr int kHalfD = D / 2;             // output columns per softmax thread
};

// Warp roles: 0 TMA producer; 1 MMA issuer; 4..11 softmax, two threads per query row (warp w
// reads TMEM lane quarter w % 4; warps 4-7 take key columns [0, 32) of each tile and output
// columns [0, D/2), warps 8-11 the other halves), exchanging row max and sum through shared
// memory (each pair of warps that shares a lane quarter on its own named barrier).  S is
// double-buffered in TMEM and K in shared memory: Q.K^T runs up to two tiles ahead, and the P.V
// of tile j runs on the tensor cores while the softmax of tile j + 1 is computed.
template <int D>
__global__ void __launch_bounds__(kAttnTcThreads, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap map_qhi, const __grid_constant__ CUtensorMap map_qlo,
                        const __grid_constant__ CUtensorMap map_khi, const __grid_constant__ CUtensorMap map_klo,
                        const __grid_constant__ CUtensorMap map_vhi, const __grid_constant__ CUtensorMap map_vlo,
                        AttnTcParams p) {
    using S = AttnShape<D>;
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t bars[11];
    __shared__ uint32_t tmem_slot;
    __shared__ int abort_flag;
    __shared__ float red_max[2][AQ], red_sum[2][AQ];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* base_ptr = smem_raw + (base - raw);
    const uint32_t b0 = smem_u32(bars);
    // k_full / k_empty of K slot b: b0 + 8 / b0 + 16 for slot 0, b0 + 72 / b0 + 80 for slot 1
    auto k_full = [&](int b) { return b ? b0 + 72 : b0 + 8; };
    auto k_empty = [&](int b) { return b ? b0 + 80 : b0 + 16; };
    const uint32_t q_full = b0, v_full = b0 + 24, v_empty = b0 + 32,
                   p_full = b0 + 40, pv_full = b0 + 48, s_full0 = b0 + 56;  // s_full[2] at 56, 64
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

    // Heavy (late) query tiles first: causal tiles near the end see the most keys.
    const int qt = p.q_tiles - 1 - (int)blockIdx.x;
    const uint64_t head = blockIdx.y;
    const uint64_t kvh = head / p.group;
    const uint64_t q0 = (uint64_t)qt * AQ;
    const uint64_t q_last = min(q0 + AQ, p.seq_len) - 1;
    // Keys this tile can admit: [key_lo, key_hi).
    const uint64_t key_hi = p.causal ? min(p.kv_seq_len, p.qpos0 + q_last + 1) : p.kv_seq_len;
    uint64_t key_lo = 0;
    if (p.window >= 0) {
        const uint64_t back = p.window > 0 ? (uint64_t)p.window - 1 : 0;
        const uint64_t pos = p.qpos0 + q0;
        key_lo = pos > back ? pos - back : 0;
    }
    const uint64_t kv0 = (key_lo / AKV) * AKV;
    const int n_kv = key_hi > kv0 ? (int)((key_hi - kv0 + AKV - 1) / AKV) : 0;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        mbar_init(k_full(0), 1);
        mbar_init(k_empty(0), 1);
        mbar_init(k_full(1), 1);
        mbar_init(k_empty(1), 1);
        mbar_init(v_full, 1);
        mbar_init(v_empty, 1);
        mbar_init(p_full, 8);  // the softmax warps
        mbar_init(pv_full, 1);
        mbar_init(s_full0, 1);
        mbar_init(s_full0 + 8, 1);
        abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&tmem_slot), S::kTmemCols);
        tmem_relinquish();
    }
    pdl_enter();  // after the TMEM allocation, as every tensor-memory kernel here does
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;

    if (warp == 0) {
        // ---- TMA producer ----------------------------------------------------------------------
        if (lane == 0 && n_kv > 0) {
            mbar_arrive_expect_tx(q_full, 2 * S::kQ);
            for (int a = 0; a < D / 64; a++) {
                tma_load_2d(base + S::kOffQ + a * S::kQAtom, &map_qhi, q_full, (int)(head * D + a * 64), (int)q0);
                tma_load_2d(base + S::kOffQ + S::kQ + a * S::kQAtom, &map_qlo, q_full, (int)(head * D + a * 64), (int)q0);
            }
            // K of tile t into slot t % 2, once the scores of tile t - 2 (the slot's last user)
            // are done: K runs one tile ahead of V.
            auto load_k = [&](int t) -> bool {
                const int b = t & 1;
                if (t >= 2 && !mbar_wait(k_empty(b), (uint32_t)((t - 2) >> 1) & 1u)) return false;
                const int key = (int)(kv0 + (uint64_t)t * AKV);
                const uint32_t slot = base + S::kOffK + (uint32_t)(b * 2 * S::kK);
                mbar_arrive_expect_tx(k_full(b), 2 * S::kK);
                for (int a = 0; a < D / 64; a++) {
                    tma_load_2d(slot + a * S::kKAtom, &map_khi, k_full(b), (int)(kvh * D + a * 64), key);
                    tma_load_2d(slot + S::kK + a * S::kKAtom, &map_klo, k_full(b), (int)(kvh * D + a * 64), key);
                }
                return true;
            };
            bool ok = load_k(0);
            for (int j = 0; j < n_kv && ok; j++) {
                const int key0 = (int)(kv0 + (uint64_t)j * AKV);
                const uint32_t ph = (uint32_t)(j - 1) & 1u;
                if (j + 1 < n_kv && !load_k(j + 1)) {
                    ok = false;
                    break;
                }
                if (j > 0 && !mbar_wait(v_empty, ph)) {
                    abort_flag = 1;
                    atomicExch(p.error, 1);
                    break;
                }
                mbar_arrive_expect_tx(v_full, 2 * S::kV);
                tma_load_2d(base + S::kOffV, &map_vhi, v_full, key0, (int)(kvh * D));
                tma_load_2d(base + S::kOffV + S::kV, &map_vlo, v_full, key0, (int)(kvh * D));
            }
            if (!ok) {
                abort_flag = 1;
                atomicExch(p.error, 1);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---- MMA issuer --------------------------------------------------------------------------
        if (lane == 0 && n_kv > 0) {
            constexpr uint32_t idesc_s = idesc_bf16(AQ, AKV);
            constexpr uint32_t idesc_o = idesc_bf16(AQ, D);
            const uint32_t tO = tmem + S::kColPV;
            // S(j) = Q K(j)^T into TMEM columns [64 * (j % 2), +64), then frees K's buffer.
            auto issue_s = [&](int j) -> bool {
                if (!mbar_wait(k_full(j & 1), (uint32_t)(j >> 1) & 1u)) return false;
                tc_fence_after();
                const uint32_t tS = tmem + (uint32_t)(j & 1) * AKV;
#pragma unroll
                for (int kk = 0; kk < D / 16; kk++) {
                    const uint32_t off = (uint32_t)(kk % 4) * 32;
                    const uint32_t qa = base + S::kOffQ + (kk / 4) * S::kQAtom + off;
                    const uint32_t kb = base + S::kOffK + (uint32_t)((j & 1) * 2 * S::kK) + (kk / 4) * S::kKAtom + off;
                    const uint64_t qhi = desc_k_sw128(qa), qlo = desc_k_sw128(qa + S::kQ);
                    const uint64_t khi = desc_k_sw128(kb), klo = desc_k_sw128(kb + S::kK);
                    mma_bf16(tS, qlo, khi, idesc_s, kk > 0 ? 1u : 0u);
                    mma_bf16(tS, qhi, klo, idesc_s, 1u);
                    mma_bf16(tS, qhi, khi, idesc_s, 1u);
                }
                tc_commit(k_empty(j & 1));
                tc_commit(s_full0 + 8u * (uint32_t)(j & 1));
                return true;
            };
            // S runs two tiles ahead: S(j + 2) reuses S(j)'s TMEM columns, which are free once
            // P(j) is written; P.V(j) is issued first so the softmax of tile j + 1 (whose S is
            // ready) overlaps it.
            bool ok = mbar_wait(q_full, 0) && issue_s(0) && (n_kv < 2 || issue_s(1));
            for (int j = 0; j < n_kv && ok; j++) {
                const uint32_t ph = (uint32_t)j & 1u;
                if (!mbar_wait(p_full, ph) || !mbar_wait(v_full, ph)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                // P.V over the tile's 64 keys in steps of 16
#pragma unroll
                for (int kk = 0; kk < AKV / 16; kk++) {
                    const uint32_t off = (uint32_t)kk * 32;
                    const uint32_t pa = base + S::kOffP + off;
                    const uint32_t vb = base + S::kOffV + off;
                    const uint64_t phi = desc_k_sw128(pa), plo = desc_k_sw128(pa + S::kP);
                    const uint64_t vhi = desc_k_sw128(vb), vlo = desc_k_sw128(vb + S::kV);
                    mma_bf16(tO, plo, vhi, idesc_o, kk > 0 ? 1u : 0u);
                    mma_bf16(tO, phi, vlo, idesc_o, 1u);
                    mma_bf16(tO, phi, vhi, idesc_o, 1u);
                }
                tc_commit(v_empty);
                tc_commit(pv_full);
                if (j + 2 < n_kv && !issue_s(j + 2)) {
                    ok = false;
                    break;
                }
            }
            if (!ok) {
                abort_flag = 1;
                atomicExch(p.error, 1);
            }
        }
        __syncwarp();
    } else if (warp >= 4) {
        // ---- softmax / output: two threads per query row --------------------------------------
        constexpr float kLog2e = 1.4426950408889634f;
        const int qq = warp % 4;
        const int hf = (warp - 4) / 4;  // which half of the key / output columns
        const int r = qq * 32 + lane;
        const uint64_t qi = q0 + r;
        const bool live = qi < p.seq_len;
        const uint64_t qpos = p.qpos0 + qi;
        const uint64_t row_hi = live ? (p.causal ? min(p.kv_seq_len, qpos + 1) : p.kv_seq_len) : 0;
        uint64_t row_lo = 0;
        if (p.window >= 0) {
            const uint64_t back = p.window > 0 ? (uint64_t)p.window - 1 : 0;
            row_lo = qpos > back ? qpos - back : 0;
            if (row_lo > row_hi) row_lo = row_hi;
        }
        const float scale2 = p.scale * kLog2e;  // scores in log2 units
        // The two threads of a row are in warps qq + 4 and qq + 8: those two warps meet on
        // named barrier 1 + qq (64 threads) to exchange the row's max and sum.
        auto pair_sync = [&]() { asm volatile("bar.sync %0, 64;" ::"r"(1 + qq) : "memory"); };
        const uint32_t lane_base = tmem + ((uint32_t)(qq * 32) << 16);
        float o[S::kHalfD];
#pragma unroll
        for (int d = 0; d < S::kHalfD; d++) o[d] = 0.0f;
        float m = __int_as_float(0xff800000), l = 0.0f;
        uint8_t* p_hi = base_ptr + S::kOffP + r * 128;
        uint8_t* p_lo = p_hi + S::kP;
        // Every softmax warp runs every iteration (the named barriers below need all 256
        // threads); a wait that times out marks the CTA failed and later waits are skipped.
        bool failed = false;
        // O <- O * keep + P.V(t): tile t's P.V, read from TMEM once its MMA has completed.
        auto fold_pv = [&](int t, float keep) {
            if (!failed && !mbar_wait(pv_full, (uint32_t)t & 1u)) failed = true;
            failed = __any_sync(0xffffffffu, failed);
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < S::kHalfD; c += 32) {
                float pv[32];
                tmem_ld32(lane_base + S::kColPV + (uint32_t)(hf * S::kHalfD + c), pv);
                tc_wait_ld();
#pragma unroll
                for (int e = 0; e < 32; e++) o[c + e] = o[c + e] * keep + pv[e];
            }
        };
        // The softmax of tile j runs while tile j - 1's P.V is on the tensor cores; that P.V is
        // folded in only then (with its own keep factor), before P(j) replaces P(j - 1).
        float keep_prev = 0.0f;
        for (int j = 0; j < n_kv; j++) {
            if (!failed && !mbar_wait(s_full0 + 8u * (uint32_t)(j & 1), (uint32_t)(j >> 1) & 1u)) failed = true;
            failed = __any_sync(0xffffffffu, failed);
            tc_fence_after();
            float s[32];
            tmem_ld32(lane_base + (uint32_t)(j & 1) * AKV + (uint32_t)hf * 32, s);
            tc_wait_ld();
            const uint64_t key0 = kv0 + (uint64_t)j * AKV + (uint64_t)hf * 32;
            float tmax = __int_as_float(0xff800000);
            if (key0 >= row_lo && key0 + 32 <= row_hi) {  // interior: every key admitted
#pragma unroll
                for (int c = 0; c < 32; c++) {
                    s[c] *= scale2;
                    tmax = fmaxf(tmax, s[c]);
                }
            } else {
#pragma unroll
                for (int c = 0; c < 32; c++) {
                    const uint64_t key = key0 + c;
                    s[c] = (key >= row_lo && key < row_hi) ? s[c] * scale2 : __int_as_float(0xff800000);
                    tmax = fmaxf(tmax, s[c]);
                }
            }
            red_max[hf][r] = tmax;
            pair_sync();
            const float m_new = fmaxf(m, fmaxf(red_max[0][r], red_max[1][r]));
            float alpha = 0.0f, psum = 0.0f;
            if (m_new != __int_as_float(0xff800000)) {
                alpha = m == __int_as_float(0xff800000) ? 0.0f : exp2f(m - m_new);
#pragma unroll
                for (int c = 0; c < 32; c++) {
                    s[c] = exp2f(s[c] - m_new);  // masked (-inf) scores give 0
                    psum += s[c];
                }
            } else {
#pragma unroll
                for (int c = 0; c < 32; c++) s[c] = 0.0f;
            }
            red_sum[hf][r] = psum;
            pair_sync();
            const float l_new = l * alpha + (red_sum[0][r] + red_sum[1][r]);
            const float inv = l_new > 0.0f ? 1.0f / l_new : 0.0f;
            const float keep = l_new > 0.0f ? (l * alpha) * inv : 0.0f;
            if (j > 0) fold_pv(j - 1, keep_prev);
            // P / l_new as bf16 hi / lo: 16-byte chunk c of row r lives at chunk (c ^ (r % 8)).
            // P(j) overwrites P(j - 1), whose P.V has completed (fold_pv waited for it).
#pragma unroll
            for (int cc = 0; cc < 4; cc++) {
                const int c = hf * 4 + cc;
                uint32_t h[4], lo4[4];
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const float x0 = s[cc * 8 + 2 * e] * inv, x1 = s[cc * 8 + 2 * e + 1] * inv;
                    const __nv_bfloat162 hb = __floats2bfloat162_rn(x0, x1);
                    const float2 hf2 = __bfloat1622float2(hb);
                    const __nv_bfloat162 lb = __floats2bfloat162_rn(x0 - hf2.x, x1 - hf2.y);
                    h[e] = *reinterpret_cast<const uint32_t*>(&hb);
                    lo4[e] = *reinterpret_cast<const uint32_t*>(&lb);
                }
                const int sw = (c ^ (r & 7)) * 16;
                *reinterpret_cast<uint4*>(p_hi + sw) = make_uint4(h[0], h[1], h[2], h[3]);
                *reinterpret_cast<uint4*>(p_lo + sw) = make_uint4(lo4[0], lo4[1], lo4[2], lo4[3]);
            }
            fence_proxy_async();  // the P writes are read by tcgen05.mma
            tc_fence_before();    // ... and the P.V read above precedes the next P.V's write
            mbar_arrive_warp(p_full);
            keep_prev = keep;
            m = m_new;
            l = l_new;
        }
        if (n_kv > 0) fold_pv(n_kv - 1, keep_prev);
        if (failed) atomicExch(p.error, 1);
        if (live) {
            float* orow = p.out + qi * p.out_dim + head * D + hf * S::kHalfD;
#pragma unroll
            for (int d = 0; d < S::kHalfD; d += 4)
                *reinterpret_cast<float4*>(orow + d) = make_float4(o[d], o[d + 1], o[d + 2], o[d + 3]);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, S::kTmemCols);
    }
}

// 2^x by the SFU's approximate exponential (relative error about 2^-22; -inf gives +0; results
// below 2^-126 flush to zero -- weights that small do not move an f32 softmax sum).
__device__ __forceinline__ float ex2_sfu(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// ---- two query tiles per CTA; P and the output in tensor memory --------------------------------
// A CTA serves 256 queries of one head as two 128-row tiles that share every K and V tile it
// loads.  Tensor memory holds, per query tile t, two 64-key score buffers (columns 256 t and
// 256 t + 64) and the output accumulator (256 t + 128, D columns).  Warp 0 loads with TMA, warp
// 1 issues the MMAs, warps 4-7 (tile 0) and 8-11 (tile 1) -- one query row per thread, one
// tensor-memory lane quarter per warp -- first split their query rows into the Q tiles, then run
// the softmax.  The softmax writes P as bf16 hi / lo
// over the scores it has just read (two bf16 per column), and the P.V MMA reads P from tensor
// memory as its A operand and accumulates into the output there: no P round trip through shared
// memory and no per-tile fold of P.V into registers.  The MMA warp issues S(j + 2) of a tile
// right after that tile's P.V(j) (tensor-core operations of one thread run in order), so the
// score buffer P(j) lived in is rewritten only after P.V(j) has read it.
//
// The output accumulates unnormalised (P = 2^(s - m), s and m in log2 units, with a reference max
// m that moves only when a tile's row max exceeds it by more than 12, a factor of 2^12; the
// output and sum are then rescaled in tensor memory) and is divided by the sum at the end.  When |V| is large enough for that sum to
// overflow (the split pass records max |v|), every tile instead rescales the output so that it
// stays a weighted mean of V rows (the reference's overflow-safety invariant).
// The reference max of the unnormalised form trails the true row max by at most 12 in log2 units:
// weights stay below 2^12 = 4096, and the output is rescaled only when a tile passes it by more.
constexpr int kAttnLazyLog2 = 12;

struct Attn2Params {
    float* out;
    uint64_t seq_len, kv_seq_len, group, out_dim;
    int causal;
    int64_t window;  // -1: none
    uint64_t qpos0;  // position of query 0
    float scale;
    int q_pairs;            // CTAs per head: 256 queries each
    const float* q;         // f32 queries [seq_len, q_ld]: each query row is split by its own thread
    uint64_t q_ld;
    const unsigned* vmax;   // bits of max |v| over V (written by the split pass)
    unsigned safe_bits;     // from this max on: the weighted-mean form
    int* error;
};

template <int D>
struct Attn2Shape {
    static constexpr int kQAtom = AQ * 128;          // [128 rows][64 bf16]
    static constexpr int kQ = (D / 64) * kQAtom;     // one term of one query tile
    static constexpr int kKAtom = AKV * 128;         // [64 keys][64 bf16]
    static constexpr int kK = (D / 64) * kKAtom;     // one term of a K tile
    static constexpr int kV = D * 128;               // one term of a V^T tile: [D][64 keys]
    static constexpr int kOffQ = 0;                  // [tile][term]
    static constexpr int kOffK = 4 * kQ;             // [slot][term], double-buffered
    static constexpr int kOffV = kOffK + 4 * kK;     // [term]
    static constexpr int kBytes = kOffV + 2 * kV;
    static constexpr int kSmem = kBytes + 1024;
    static constexpr uint32_t kTmemCols = 512;
    static constexpr uint32_t kColO = 128;           // within a tile's 256 columns
};

template <int D>
__global__ void __launch_bounds__(kAttnTcThreads, 1)
    attention_tc2_kernel(const __grid_constant__ CUtensorMap map_khi, const __grid_constant__ CUtensorMap map_klo,
                         const __grid_constant__ CUtensorMap map_vhi, const __grid_constant__ CUtensorMap map_vlo,
                         Attn2Params p) {
    using S = Attn2Shape<D>;
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t bars[19];
    __shared__ uint32_t tmem_slot;
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* base_ptr = smem_raw + (base - raw);
    const uint32_t b0 = smem_u32(bars);
    const uint32_t q_full = b0, v_full = b0 + 8, v_empty = b0 + 16;
    auto k_full = [&](int b) { return b0 + 24 + 8u * (uint32_t)b; };
    auto k_empty = [&](int b) { return b0 + 40 + 8u * (uint32_t)b; };
    auto s_full = [&](int t, int b) { return b0 + 56 + 8u * (uint32_t)(2 * t + b); };
    // P(j) of tile t is written on p_full(t, j % 2) and P.V(j) completes on pv_done(t, j % 2): two
    // barriers each per tile, because the softmax may run one tile ahead of the MMAs (the scores
    // are double-buffered) -- a parity wait must never meet a barrier two phases ahead of it
    auto p_full = [&](int t, int b) { return b0 + 88 + 8u * (uint32_t)(2 * t + b); };
    auto pv_done = [&](int t, int b) { return b0 + 120 + 8u * (uint32_t)(2 * t + b); };
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

    // Heavy (late) query pairs first across all heads (the grid's x runs over heads): causal
    // pairs near the end see the most keys, and CTAs start in grid order, so the light pairs fill
    // the machine's last wave instead of heavy ones.
    const int qp = p.q_pairs - 1 - (int)blockIdx.y;
    const uint64_t head = blockIdx.x;
    const uint64_t kvh = head / p.group;
    const uint64_t q0 = (uint64_t)qp * 2 * AQ;
    uint64_t key_lo = 0;
    if (p.window >= 0) {
        const uint64_t back = p.window > 0 ? (uint64_t)p.window - 1 : 0;
        const uint64_t pos = p.qpos0 + q0;
        key_lo = pos > back ? pos - back : 0;
    }
    const uint64_t kv0 = (key_lo / AKV) * AKV;
    // Key tiles each query tile reads: [kv0, its last admitted key]; the CTA loads the longer run.
    int n_t[2];
#pragma unroll
    for (int t = 0; t < 2; t++) {
        const uint64_t tq0 = q0 + (uint64_t)t * AQ;
        n_t[t] = 0;
        if (tq0 < p.seq_len) {
            const uint64_t q_last = min(tq0 + AQ, p.seq_len) - 1;
            const uint64_t key_hi = p.causal ? min(p.kv_seq_len, p.qpos0 + q_last + 1) : p.kv_seq_len;
            n_t[t] = key_hi > kv0 ? (int)((key_hi - kv0 + AKV - 1) / AKV) : 0;
        }
    }
    const int n_kv = max(n_t[0], n_t[1]);

    if (threadIdx.x == 0) {
        for (int i = 0; i < 19; i++) {
            const uint32_t bar = b0 + 8u * (uint32_t)i;
            // P: the tile's four softmax warps; Q: all eight softmax warps
            mbar_init(bar, bar >= p_full(0, 0) && bar <= p_full(1, 1) ? 4 : bar == q_full ? 8 : 1);
        }
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&tmem_slot), S::kTmemCols);
        tmem_relinquish();
    }
    pdl_enter();  // after the TMEM allocation, as every tensor-memory kernel here does
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;

    if (warp == 0) {
        // ---- TMA producer ----------------------------------------------------------------------
        if (lane == 0 && n_kv > 0) {
            // K of tile j into slot j % 2, once the scores of tile j - 2 (the slot's last user)
            // are done: K runs ahead of V.
            auto load_k = [&](int j) -> bool {
                const int b = j & 1;
                if (j >= 2 && !mbar_wait(k_empty(b), (uint32_t)((j - 2) >> 1) & 1u)) return false;
                const int key = (int)(kv0 + (uint64_t)j * AKV);
                const uint32_t slot = base + S::kOffK + (uint32_t)(b * 2 * S::kK);
                mbar_arrive_expect_tx(k_full(b), 2 * S::kK);
                for (int a = 0; a < D / 64; a++) {
                    tma_load_2d(slot + a * S::kKAtom, &map_khi, k_full(b), (int)(kvh * D + a * 64), key);
                    tma_load_2d(slot + S::kK + a * S::kKAtom, &map_klo, k_full(b), (int)(kvh * D + a * 64), key);
                }
                return true;
            };
            bool ok = load_k(0);
            for (int j = 0; j < n_kv && ok; j++) {
                if (j + 1 < n_kv && !load_k(j + 1)) {
                    ok = false;
                    break;
                }
                if (j > 0 && !mbar_wait(v_empty, (uint32_t)(j - 1) & 1u)) {
                    ok = false;
                    break;
                }
                const int key0 = (int)(kv0 + (uint64_t)j * AKV);
                mbar_arrive_expect_tx(v_full, 2 * S::kV);
                tma_load_2d(base + S::kOffV, &map_vhi, v_full, key0, (int)(kvh * D));
                tma_load_2d(base + S::kOffV + S::kV, &map_vlo, v_full, key0, (int)(kvh * D));
            }
            if (!ok) atomicExch(p.error, 1);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---- MMA issuer --------------------------------------------------------------------------
        if (lane == 0 && n_kv > 0) {
            constexpr uint32_t idesc_s = idesc_bf16(AQ, AKV);
            constexpr uint32_t idesc_o = idesc_bf16(AQ, D);
            // Shared-memory descriptors advance by (byte offset >> 4) in their start-address
            // field: the operands' descriptors are the region's base descriptor plus constants, so
            // the issuing thread spends a few adds per MMA (it shares its scheduler with two
            // softmax warps).
            const uint64_t dq0 = desc_k_sw128(base + S::kOffQ), dk0 = desc_k_sw128(base + S::kOffK);
            const uint64_t dv0 = desc_k_sw128(base + S::kOffV);
            // S_t(j) = Q_t K(j)^T into tile t's score buffer j % 2
            auto issue_s = [&](int t, int j) {
                const uint32_t tS = tmem + 256u * (uint32_t)t + (uint32_t)(j & 1) * AKV;
                const uint64_t dq = dq0 + (uint64_t)((2 * t * S::kQ) >> 4);
                const uint64_t dk = dk0 + (uint64_t)(((j & 1) * 2 * S::kK) >> 4);
#pragma unroll
                for (int kk = 0; kk < D / 16; kk++) {
                    const uint32_t off = (uint32_t)(((kk / 4) * S::kQAtom + (kk % 4) * 32) >> 4);
                    const uint32_t offk = (uint32_t)(((kk / 4) * S::kKAtom + (kk % 4) * 32) >> 4);
                    const uint64_t qhi = dq + off, qlo = qhi + (uint64_t)(S::kQ >> 4);
                    const uint64_t khi = dk + offk, klo = khi + (uint64_t)(S::kK >> 4);
                    mma_bf16(tS, qlo, khi, idesc_s, kk > 0 ? 1u : 0u);
                    mma_bf16(tS, qhi, klo, idesc_s, 1u);
                    mma_bf16(tS, qhi, khi, idesc_s, 1u);
                }
                tc_commit(s_full(t, j & 1));
            };
            bool ok = mbar_wait(q_full, 0);
            for (int j = 0; j < min(2, n_kv) && ok; j++) {
                ok = mbar_wait(k_full(j), 0);
                if (!ok) break;
                tc_fence_after();
                for (int t = 0; t < 2; t++)
                    if (j < n_t[t]) issue_s(t, j);
                tc_commit(k_empty(j));
            }
            for (int j = 0; j < n_kv && ok; j++) {
                if (!mbar_wait(v_full, (uint32_t)j & 1u)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                bool k_ready = false;
                for (int t = 0; t < 2 && ok; t++) {
                    if (j < n_t[t]) {
                        if (!mbar_wait(p_full(t, j & 1), (uint32_t)(j >> 1) & 1u)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        // O_t += P_t(j) V(j): P's hi / lo terms from tensor memory (32 columns
                        // each, two bf16 per column), V^T's from shared memory
                        const uint32_t tP = tmem + 256u * (uint32_t)t + (uint32_t)(j & 1) * AKV;
                        const uint32_t tO = tmem + 256u * (uint32_t)t + S::kColO;
#pragma unroll
                        for (int kk = 0; kk < AKV / 16; kk++) {
                            const uint64_t vhi = dv0 + (uint64_t)(kk * 2), vlo = vhi + (uint64_t)(S::kV >> 4);
                            const uint32_t ahi = tP + (uint32_t)kk * 8, alo = ahi + 32;
                            mma_bf16_ts(tO, alo, vhi, idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
                            mma_bf16_ts(tO, ahi, vlo, idesc_o, 1u);
                            mma_bf16_ts(tO, ahi, vhi, idesc_o, 1u);
                        }
                        tc_commit(pv_done(t, j & 1));
                    }
                    if (t == 1) tc_commit(v_empty);
                    if (j + 2 < n_t[t]) {
                        if (!k_ready) {
                            if (!mbar_wait(k_full(j & 1), (uint32_t)((j + 2) >> 1) & 1u)) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                            k_ready = true;
                        }
                        issue_s(t, j + 2);
                    }
                }
                if (ok && j + 2 < n_kv) tc_commit(k_empty(j & 1));
            }
            if (!ok) atomicExch(p.error, 1);
        }
        __syncwarp();
    } else if (warp >= 4) {
        // ---- softmax: one query row per thread ---------------------------------------------------
        constexpr float kLog2e = 1.4426950408889634f;
        const float kNegInf = __int_as_float(0xff800000);
        const int t = (warp - 4) / 4, qq = warp % 4;
        const int r = qq * 32 + lane;
        const uint64_t qi = q0 + (uint64_t)t * AQ + r;
        const bool live = qi < p.seq_len;
        {
            // This warp's 32 query rows (the rows its lanes own) as bf16 hi / lo terms in the MMA's
            // K-major layout: 64 columns per 128-byte row of an atom, 16-byte chunk c at position
            // c ^ (row % 8); zeros past the sequence.  (Each query row belongs to this CTA alone,
            // so it is split here rather than by a pass over Q.)  The warp reads one row per load,
            // each lane D / 32 consecutive columns, so a load touches the row's own cache lines
            // only; all 32 rows' loads are in flight before the first is split.
            constexpr int V = D / 32;  // columns per lane: 4 (D = 128) or 2 (D = 64)
            using Vec = typename std::conditional<V == 4, float4, float2>::type;
            const uint64_t row0 = q0 + (uint64_t)t * AQ + (uint64_t)qq * 32;
            Vec xv[32];
#pragma unroll
            for (int i = 0; i < 32; i++) {
                const bool row_live = row0 + i < p.seq_len;
                const float* src = p.q + (row_live ? row0 + i : 0) * p.q_ld + head * D + lane * V;
                if (row_live) xv[i] = __ldg(reinterpret_cast<const Vec*>(src));
                else xv[i] = Vec{};
            }
            uint8_t* qt0 = base_ptr + S::kOffQ + (size_t)(2 * t) * S::kQ;
            const int e0 = lane * V;  // this lane's first column
            const int a = e0 / 64, c = (e0 % 64) / 8, byte = (e0 % 8) * 2;
#pragma unroll
            for (int i = 0; i < 32; i++) {
                const int rr = qq * 32 + i;
                const size_t off = (size_t)a * S::kQAtom + (size_t)rr * 128 + (size_t)((c ^ (rr & 7)) * 16 + byte);
                const float* xs = reinterpret_cast<const float*>(&xv[i]);
                uint16_t h[V], lo[V];
#pragma unroll
                for (int e = 0; e < V; e++) split_bf16(xs[e], h[e], lo[e]);
                if constexpr (V == 4) {
                    *reinterpret_cast<uint2*>(qt0 + off) = make_uint2(pack_bf16(h[0], h[1]), pack_bf16(h[2], h[3]));
                    *reinterpret_cast<uint2*>(qt0 + S::kQ + off) = make_uint2(pack_bf16(lo[0], lo[1]), pack_bf16(lo[2], lo[3]));
                } else {
                    *reinterpret_cast<uint32_t*>(qt0 + off) = pack_bf16(h[0], h[1]);
                    *reinterpret_cast<uint32_t*>(qt0 + S::kQ + off) = pack_bf16(lo[0], lo[1]);
                }
            }
            fence_proxy_async();  // the generic-proxy writes are read by tcgen05.mma
            mbar_arrive_warp(q_full);
        }
        const uint64_t qpos = p.qpos0 + qi;
        const uint64_t row_hi = live ? (p.causal ? min(p.kv_seq_len, qpos + 1) : p.kv_seq_len) : 0;
        uint64_t row_lo = 0;
        if (p.window >= 0) {
            const uint64_t back = p.window > 0 ? (uint64_t)p.window - 1 : 0;
            row_lo = qpos > back ? qpos - back : 0;
            if (row_lo > row_hi) row_lo = row_hi;
        }
        const float scale2 = p.scale * kLog2e;  // scores in log2 units
        const bool pos_scale = scale2 > 0.0f;
        const float sc = pos_scale ? scale2 : 1.0f;  // the factor left for after the max
        constexpr float kLazy = (float)kAttnLazyLog2;
        const bool safe = *p.vmax >= p.safe_bits;
        const uint32_t lane_base = tmem + ((uint32_t)(qq * 32) << 16) + 256u * (uint32_t)t;
        const int n = n_t[t];
        float m = kNegInf, l = 0.0f;
        bool failed = false;
        // O *= f for this thread's row (warp-collective), once P.V(j - 1) has completed
        auto rescale_o = [&](int j, float f) {
            if (!mbar_wait(pv_done(t, (j - 1) & 1), (uint32_t)((j - 1) >> 1) & 1u)) failed = true;
            failed = __any_sync(0xffffffffu, failed);
            if (failed) return;
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < D; c += 32) {
                float o[32];
                tmem_ld32(lane_base + S::kColO + (uint32_t)c, o);
                tc_wait_ld();
                uint32_t u0[16], u1[16];
#pragma unroll
                for (int e = 0; e < 16; e++) {
                    u0[e] = __float_as_uint(o[e] * f);
                    u1[e] = __float_as_uint(o[16 + e] * f);
                }
                tmem_st16(lane_base + S::kColO + (uint32_t)c, u0);
                tmem_st16(lane_base + S::kColO + (uint32_t)c + 16, u1);
            }
            tc_wait_st();
        };
        for (int j = 0; j < n; j++) {
            if (!mbar_wait(s_full(t, j & 1), (uint32_t)(j >> 1) & 1u)) failed = true;
            failed = __any_sync(0xffffffffu, failed);
            if (failed) break;
            tc_fence_after();
            const uint32_t tS = lane_base + (uint32_t)(j & 1) * AKV;
            float s[64];
            tmem_ld32(tS, s);
            tmem_ld32(tS + 32, s + 32);
            tc_wait_ld();
            const uint64_t key0 = kv0 + (uint64_t)j * AKV;
            // eight independent running maxima / sums: short dependency chains
            float mx[8];
#pragma unroll
            for (int g = 0; g < 8; g++) mx[g] = kNegInf;
            // The row max of the raw scores (a positive scale keeps their order; any other
            // scale is applied first), in log2 units after one multiply.
            if (!pos_scale)
#pragma unroll
                for (int c = 0; c < 64; c++) s[c] *= scale2;
            if (key0 >= row_lo && key0 + AKV <= row_hi) {  // interior: every key admitted
#pragma unroll
                for (int c = 0; c < 64; c++) mx[c & 7] = fmaxf(mx[c & 7], s[c]);
            } else {
#pragma unroll
                for (int c = 0; c < 64; c++) {
                    const uint64_t key = key0 + c;
                    s[c] = (key >= row_lo && key < row_hi) ? s[c] : kNegInf;
                    mx[c & 7] = fmaxf(mx[c & 7], s[c]);
                }
            }
            const float tmax = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                                     fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))) * sc;
            // weights 2^(s sc - ref) (one FMA and the SFU) for a finite reference; none while the
            // row has no admitted key
            auto weights = [&](float ref) {
                float ps[8];
#pragma unroll
                for (int g = 0; g < 8; g++) ps[g] = 0.0f;
                if (ref != kNegInf) {
#pragma unroll
                    for (int c = 0; c < 64; c++) {
                        s[c] = ex2_sfu(fmaf(s[c], sc, -ref));  // masked (-inf) keys give +0
                        ps[c & 7] += s[c];
                    }
                } else {
#pragma unroll
                    for (int c = 0; c < 64; c++) s[c] = 0.0f;
                }
                return ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
            };
            float pmul = 1.0f, f = 1.0f, a = 1.0f;
            bool need = false;
            const float m_old = m;
            if (!safe) {
                // the reference max moves only when this tile's passes it by more than 2^kLazy
                need = tmax != kNegInf && (m == kNegInf || tmax > m + kLazy);
                if (need) {
                    f = m == kNegInf ? 0.0f : ex2_sfu(m - tmax);
                    need = m != kNegInf;  // an output that holds only zero weights needs no rescale
                    m = tmax;
                    l *= f;
                }
            } else {
                m = fmaxf(m, tmax);
                a = m_old == kNegInf ? 0.0f : ex2_sfu(m_old - m);
            }
            const float psum = weights(m);
            if (!safe) {
                l += psum;
            } else {
                // the output stays a weighted mean of V rows: O <- O (l a / l_new) + (P / l_new) V
                const float l_new = l * a + psum;
                pmul = l_new > 0.0f ? 1.0f / l_new : 0.0f;
                f = l_new > 0.0f ? (l * a) * pmul : 0.0f;
                need = true;
                l = l_new;
            }
            if (j > 0 && __any_sync(0xffffffffu, need)) {
                rescale_o(j, need ? f : 1.0f);
                if (failed) break;
            }
            // P as bf16 hi / lo over the scores just read: 64 keys, two per column; hi in
            // columns [0, 32), lo in [32, 64) (the lower key in the low half)
            if (safe)
#pragma unroll
                for (int c = 0; c < 64; c++) s[c] *= pmul;
            uint32_t ph[32], pl[32];
#pragma unroll
            for (int c = 0; c < 32; c++) {
                const float x0 = s[2 * c], x1 = s[2 * c + 1];
                const __nv_bfloat162 hb = __floats2bfloat162_rn(x0, x1);
                const float2 hf2 = __bfloat1622float2(hb);
                const __nv_bfloat162 lb = __floats2bfloat162_rn(x0 - hf2.x, x1 - hf2.y);
                ph[c] = *reinterpret_cast<const uint32_t*>(&hb);
                pl[c] = *reinterpret_cast<const uint32_t*>(&lb);
            }
            tmem_st16(tS, *reinterpret_cast<const uint32_t(*)[16]>(ph));
            tmem_st16(tS + 16, *reinterpret_cast<const uint32_t(*)[16]>(ph + 16));
            tmem_st16(tS + 32, *reinterpret_cast<const uint32_t(*)[16]>(pl));
            tmem_st16(tS + 48, *reinterpret_cast<const uint32_t(*)[16]>(pl + 16));
            tc_wait_st();
            tc_fence_before();
            mbar_arrive_warp(p_full(t, j & 1));
        }
        // ---- the output row: O / l (or the weighted mean as it stands) ---------------------------
        bool have = false;
        if (n > 0 && !failed) {
            if (!mbar_wait(pv_done(t, (n - 1) & 1), (uint32_t)((n - 1) >> 1) & 1u)) failed = true;
            failed = __any_sync(0xffffffffu, failed);
            have = !failed;
        }
        if (failed) atomicExch(p.error, 1);
        const float fin = safe ? 1.0f : (l > 0.0f ? 1.0f / l : 0.0f);
        if (have) tc_fence_after();
        // The output rows leave through shared memory.  Each thread writes its row into its warp's
        // staging area -- this tile's query terms, which no MMA reads once P.V of its last key
        // tile has completed -- with 16-byte chunk k of row i at position k ^ i; then the warp
        // stores one row per instruction, each lane 16 consecutive bytes (coalesced).
        constexpr int kChunks = D / 4;               // 16-byte chunks per row
        constexpr int kRowsPerStore = 32 / kChunks;  // rows one warp store covers
        uint8_t* stage = base_ptr + S::kOffQ + (size_t)(2 * t) * S::kQ + (size_t)qq * (32 * D * 4);
        fence_proxy_async();  // after the MMAs' reads of this area, before generic writes
#pragma unroll
        for (int c = 0; c < D; c += 32) {
            float o[32];
            if (have) {
                tmem_ld32(lane_base + S::kColO + (uint32_t)c, o);
                tc_wait_ld();
            } else {
#pragma unroll
                for (int e = 0; e < 32; e++) o[e] = 0.0f;
            }
#pragma unroll
            for (int e = 0; e < 32; e += 4) {
                const int k = (c + e) / 4;
                *reinterpret_cast<float4*>(stage + (size_t)lane * (D * 4) + (size_t)(((k ^ lane) % kChunks) * 16)) =
                    make_float4(o[e] * fin, o[e + 1] * fin, o[e + 2] * fin, o[e + 3] * fin);
            }
        }
        __syncwarp();
        const uint64_t row0 = q0 + (uint64_t)t * AQ + (uint64_t)qq * 32;
#pragma unroll 4
        for (int i0 = 0; i0 < 32; i0 += kRowsPerStore) {
            const int i = i0 + lane / kChunks, k = lane % kChunks;
            const float4 v = *reinterpret_cast<const float4*>(stage + (size_t)i * (D * 4) + (size_t)(((k ^ i) % kChunks) * 16));
            if (row0 + i < p.seq_len)
                *reinterpret_cast<float4*>(p.out + (row0 + i) * p.out_dim + head * D + 4 * k) = v;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, S::kTmemCols);
    }
}

PFN_cuTensorMapEncodeTiled_v12000 attn_encode_fn() {
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

// bf16 [rows, cols] (row stride ld elements), box [box_rows, 64] with 128-byte swizzle.
mg_status bf16_map(CUtensorMap* map, const uint16_t* ptr, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows) {
    auto fn = attn_encode_fn();
    if (!fn) return fail(MG_DRIVER_FAILED, "the driver does not provide cuTensorMapEncodeTiled");
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld * 2};
    cuuint32_t box[2] = {64, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(ptr), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(MG_DRIVER_FAILED, "encoding a TMA descriptor failed (CUresult %d)", (int)r);
    return MG_OK;
}

inline unsigned grid_for_n(const Device* d, uint64_t items) {
    uint64_t want = (items + 255) / 256, cap = (uint64_t)d->sm_count * 8;
    return (unsigned)(want < 1 ? 1 : want > cap ? cap : want);
}

template <int D>
mg_status launch_attention_tc(Device* d, const k::AttentionArgs& a, const CUtensorMap* maps, int q_tiles) {
    using S = AttnShape<D>;
    static_assert(S::kSmem <= 227 * 1024, "shared memory budget");
    static bool configured[64] = {false};
    if (!configured[d->ordinal & 63]) {
        MG_CUDA(cudaFuncSetAttribute(attention_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmem),
                "configuring the attention kernel");
        configured[d->ordinal & 63] = true;
    }
    AttnTcParams p;
    p.out = a.out;
    p.seq_len = a.seq_len;
    p.kv_seq_len = a.kv_seq_len;
    p.group = a.head_count / a.kv_head_count;
    p.out_dim = a.head_count * a.value_dim;
    p.causal = a.causal;
    p.window = a.window;
    p.qpos0 = a.query_position_offset;
    p.scale = a.scale;
    p.q_tiles = q_tiles;
    p.error = d->flags + 2;
    dim3 grid((unsigned)q_tiles, (unsigned)a.head_count);
    enqueue(d, attention_tc_kernel<D>, grid, kAttnTcThreads, S::kSmem, maps[0], maps[1], maps[2], maps[3], maps[4],
                                                                          maps[5], p);
    return launched(d, "tensor-core attention launch");
}

template <int D>
mg_status launch_attention_tc2(Device* d, const k::AttentionArgs& a, const CUtensorMap* maps, const unsigned* vmax) {
    using S = Attn2Shape<D>;
    static_assert(S::kSmem <= 227 * 1024 - 256, "shared memory budget");
    static bool configured[64] = {false};
    if (!configured[d->ordinal & 63]) {
        MG_CUDA(cudaFuncSetAttribute(attention_tc2_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmem),
                "configuring the attention kernel");
        configured[d->ordinal & 63] = true;
    }
    Attn2Params p;
    p.out = a.out;
    p.seq_len = a.seq_len;
    p.kv_seq_len = a.kv_seq_len;
    p.group = a.head_count / a.kv_head_count;
    p.out_dim = a.head_count * a.value_dim;
    p.causal = a.causal;
    p.window = a.window;
    p.qpos0 = a.query_position_offset;
    p.scale = a.scale;
    p.q_pairs = (int)((a.seq_len + 2 * AQ - 1) / (2 * AQ));
    p.q = a.q;
    p.q_ld = a.q_model_dim;
    p.vmax = vmax;
    // The unnormalised sum stays below n_keys * 2^kAttnLazyLog2 * max |v|: the weighted-mean
    // form from max |v| >= 2^(118 - kAttnLazyLog2 - ceil(log2 n_keys)), keeping 2^10 of headroom
    // below the f32 limit.
    int lg = 0;
    while (lg < 40 && (1ull << lg) < a.kv_seq_len) lg++;
    const int e = 118 - kAttnLazyLog2 - lg;
    p.safe_bits = (unsigned)(e + 127) << 23;
    p.error = d->flags + 2;
    dim3 grid((unsigned)a.head_count, (unsigned)p.q_pairs);
    enqueue(d, attention_tc2_kernel<D>, grid, kAttnTcThreads, S::kSmem, maps[2], maps[3], maps[4], maps[5], p);
    return launched(d, "tensor-core attention launch");
}

}  // namespace

namespace k {

bool attention_tc_eligible(const AttentionArgs& a) {
    const bool aligned = ((reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.k) |
                           reinterpret_cast<uintptr_t>(a.v) | reinterpret_cast<uintptr_t>(a.out)) & 15) == 0;
    return aligned && (a.head_dim == 64 || a.head_dim == 128) && a.value_dim == a.head_dim &&
           a.q_model_dim == a.head_count * a.head_dim && a.kv_model_dim == a.kv_head_count * a.head_dim &&
           a.v_model_dim == a.kv_model_dim && a.seq_len > 0 && a.kv_seq_len > 0 && a.head_count <= 65535 &&
           a.kv_seq_len < (1ull << 31) && a.q_model_dim < (1ull << 31);
}

mg_status attention_tc(Device* d, const AttentionArgs& a) {
    const uint64_t S = a.seq_len, Skv = a.kv_seq_len, qd = a.q_model_dim, kvd = a.kv_model_dim;
    const uint64_t skv_p = (Skv + 7) & ~7ull;  // V^T rows are 16-byte multiples
    static const bool one_tile_env = [] {
        const char* e = getenv("MAGNETAR_CUDA_ATTN_ONE_TILE");
        return e && atoi(e) != 0;
    }();
    // the two-tile kernel's query pairs run along the grid's y (at most 65,535 of them)
    const bool one_tile = one_tile_env || (S + 2 * AQ - 1) / (2 * AQ) > 65535;
    // Q's terms only for the one-tile kernel: the two-tile kernel splits its query rows itself.
    const size_t q_elems = one_tile ? S * qd : 0, k_elems = Skv * kvd, vt_elems = kvd * skv_p;
    uint16_t* ws = nullptr;
    const size_t terms = 2 * (q_elems + k_elems + vt_elems) * sizeof(uint16_t);
    MG_TRY(scratch(d, 4, terms + 16, (void**)&ws));
    uint16_t* qhi = ws;
    uint16_t* qlo = qhi + q_elems;
    uint16_t* khi = qlo + q_elems;
    uint16_t* klo = khi + k_elems;
    uint16_t* vhi = klo + k_elems;
    uint16_t* vlo = vhi + vt_elems;
    unsigned* vmax = reinterpret_cast<unsigned*>(reinterpret_cast<uint8_t*>(ws) + terms);
    dim3 tg((unsigned)((kvd + 63) / 64), (unsigned)((skv_p + 63) / 64));
    if (tg.y > 65535) return fail(MG_SHAPE_UNSUPPORTED, "attention has too many keys for the split pass");
    if (one_tile) {
        enqueue(d, split_bf16_rows_kernel, grid_for_n(d, q_elems / 4), 256, 0, a.q, qhi, qlo, q_elems, (unsigned*)nullptr);
        MG_TRY(launched(d, "attention split launch"));
    }
    // the K pass also zeroes the V pass's max |v| word
    enqueue(d, split_bf16_rows_kernel, grid_for_n(d, k_elems / 4), 256, 0, a.k, khi, klo, k_elems, vmax);
    MG_TRY(launched(d, "attention split launch"));
    enqueue(d, split_bf16_transpose_kernel, tg, 256, 0, a.v, Skv, kvd, vhi, vlo, skv_p, vmax);
    MG_TRY(launched(d, "attention split launch"));
    const int D = (int)a.head_dim;
    CUtensorMap maps[6];
    if (one_tile) {
        MG_TRY(bf16_map(&maps[0], qhi, S, qd, qd, AQ));
        MG_TRY(bf16_map(&maps[1], qlo, S, qd, qd, AQ));
    }
    MG_TRY(bf16_map(&maps[2], khi, Skv, kvd, kvd, AKV));
    MG_TRY(bf16_map(&maps[3], klo, Skv, kvd, kvd, AKV));
    MG_TRY(bf16_map(&maps[4], vhi, kvd, Skv, skv_p, (uint32_t)D));
    MG_TRY(bf16_map(&maps[5], vlo, kvd, Skv, skv_p, (uint32_t)D));
    if (!one_tile) return D == 64 ? launch_attention_tc2<64>(d, a, maps, vmax) : launch_attention_tc2<128>(d, a, maps, vmax);
    const int q_tiles = (int)((S + AQ - 1) / AQ);
    if (D == 64) return launch_attention_tc<64>(d, a, maps, q_tiles);
    return launch_attention_tc<128>(d, a, maps, q_tiles);
}

}  // namespace k
}  // namespace mg
