// Fused attention: softmax(Q K^T * scale) V with causal / sliding-window masks, GQA and an
// explicit key count, in one pass over K and V.
//
// Semantics follow the reference's `attention_kernel` (src/kernels.cu:1873-1959) with the
// wrapper rules of src/kernels.rs:6505-6629: query i sits at position
// (kv_seq_len - seq_len) + i; causal admits keys [lower, position + 1), a window of w keeps
// the last w of them; a query with no admitted key outputs zeros; the output is written as
// [seq, head_count * value_dimension].
//
// The tiled kernel serves BQ queries of one head per CTA with 4 threads per query (thread
// `part` owns the float4 chunks part, part + 4, ... of the head dimension), stages KT keys
// of K and V in shared memory at a time, and merges each tile into the running result
// with an online softmax.  The running output is kept as a weighted MEAN of V rows (each
// merge rescales by l_old * alpha / l_new and adds p_j / l_new times v_j), so it never
// exceeds the largest |v| -- the reference's overflow-safety invariant for large finite V
// (src/tests_conformance.rs:884-914).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "internal.h"
#include "sm100.cuh"

namespace mg {
namespace {

constexpr int BQ = 32;   // queries per CTA
constexpr int KT = 32;   // keys per shared-memory tile
constexpr int kAttnThreads = BQ * 4;

struct AttnP {
    const float* q;
    const float* k;
    const float* v;
    float* out;
    uint64_t seq_len, kv_seq_len, head_count, group, head_dim, value_dim;
    uint64_t q_model_dim, kv_model_dim, v_model_dim;
    int causal;
    int64_t window;
    uint64_t qpos0;
    float scale;
};

// Admitted keys [lo, hi) of the query at position `pos` (src/kernels.cu:1903-1913).
__device__ __forceinline__ void key_range(const AttnP& p, uint64_t pos, uint64_t& lo, uint64_t& hi) {
    hi = p.causal ? min(pos + 1, p.kv_seq_len) : p.kv_seq_len;
    lo = 0;
    if (p.window >= 0) {
        const uint64_t w = (uint64_t)p.window;
        const uint64_t back = w > 0 ? w - 1 : 0;
        lo = pos > back ? pos - back : 0;
        if (lo > hi) lo = hi;
    }
}

template <int DPT>  // float4 chunks per thread: head_dim = 16 * DPT
__global__ void __launch_bounds__(kAttnThreads) attention_tile_kernel(AttnP p) {
    pdl_enter();
    constexpr int D = 16 * DPT;
    __shared__ float4 ks[KT][D / 4];
    __shared__ float4 vs[KT][D / 4];
    const uint64_t head = blockIdx.y;
    const uint64_t kvh = head / p.group;
    const int qi = threadIdx.x / 4, part = threadIdx.x % 4;
    const uint64_t q0 = (uint64_t)blockIdx.x * BQ;
    const uint64_t query = q0 + qi;
    const bool live = query < p.seq_len;
    const uint64_t pos = p.qpos0 + (live ? query : q0);
    uint64_t lo, hi;
    key_range(p, pos, lo, hi);
    if (!live) {
        lo = hi = 0;
    }
    // Key span of the whole CTA.
    uint64_t span_lo, span_hi, tmp;
    {
        const uint64_t last = min(q0 + BQ, p.seq_len) - 1;
        key_range(p, p.qpos0 + q0, span_lo, tmp);
        key_range(p, p.qpos0 + last, tmp, span_hi);
        if (span_lo > span_hi) span_lo = span_hi;
    }

    float4 qv[DPT], ov[DPT];
    const float4* qrow = reinterpret_cast<const float4*>(p.q + (live ? query : 0) * p.q_model_dim + head * D);
#pragma unroll
    for (int i = 0; i < DPT; i++) {
        qv[i] = live ? qrow[part + 4 * i] : make_float4(0.f, 0.f, 0.f, 0.f);
        ov[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float m = __int_as_float(0xff800000), l = 0.0f;

    for (uint64_t t0 = span_lo - span_lo % KT; t0 < span_hi; t0 += KT) {
        __syncthreads();
        for (int i = threadIdx.x; i < KT * (D / 4); i += kAttnThreads) {
            const int j = i / (D / 4), c = i % (D / 4);
            const uint64_t key = t0 + j;
            float4 kk = make_float4(0.f, 0.f, 0.f, 0.f), vv = kk;
            if (key < span_hi) {
                kk = reinterpret_cast<const float4*>(p.k + key * p.kv_model_dim + kvh * D)[c];
                vv = reinterpret_cast<const float4*>(p.v + key * p.v_model_dim + kvh * D)[c];
            }
            ks[j][c] = kk;
            vs[j][c] = vv;
        }
        __syncthreads();
        float s[KT];
        float tmax = __int_as_float(0xff800000);
#pragma unroll
        for (int j = 0; j < KT; j++) {
            float dot = 0.0f;
#pragma unroll
            for (int i = 0; i < DPT; i++) {
                const float4 kk = ks[j][part + 4 * i];
                dot += qv[i].x * kk.x + qv[i].y * kk.y + qv[i].z * kk.z + qv[i].w * kk.w;
            }
            dot += __shfl_xor_sync(0xffffffffu, dot, 1);
            dot += __shfl_xor_sync(0xffffffffu, dot, 2);
            const uint64_t key = t0 + j;
            const bool ok = key >= lo && key < hi;
            s[j] = ok ? dot * p.scale : __int_as_float(0xff800000);
            tmax = fmaxf(tmax, s[j]);
        }
        const float m_new = fmaxf(m, tmax);
        if (m_new == __int_as_float(0xff800000)) continue;  // nothing admitted yet
        const float alpha = expf(m - m_new);
        float psum = 0.0f;
#pragma unroll
        for (int j = 0; j < KT; j++) {
            s[j] = expf(s[j] - m_new);
            psum += s[j];
        }
        const float l_new = l * alpha + psum;
        const float keep = (l * alpha) / l_new;
        const float inv = 1.0f / l_new;
#pragma unroll
        for (int i = 0; i < DPT; i++) {
            ov[i].x *= keep;
            ov[i].y *= keep;
            ov[i].z *= keep;
            ov[i].w *= keep;
        }
#pragma unroll
        for (int j = 0; j < KT; j++) {
            const float w = s[j] * inv;
#pragma unroll
            for (int i = 0; i < DPT; i++) {
                const float4 vv = vs[j][part + 4 * i];
                ov[i].x += w * vv.x;
                ov[i].y += w * vv.y;
                ov[i].z += w * vv.z;
                ov[i].w += w * vv.w;
            }
        }
        m = m_new;
        l = l_new;
    }
    if (!live) return;
    float4* orow = reinterpret_cast<float4*>(p.out + (query * p.head_count + head) * D);
#pragma unroll
    for (int i = 0; i < DPT; i++) orow[part + 4 * i] = ov[i];
}

// Any head / value dimension: one warp per (head, query), keys one at a time, lanes over
// dimensions, with the same weighted-mean online update.
__global__ void __launch_bounds__(256) attention_generic_kernel(AttnP p) {
    pdl_enter();
    const uint64_t warp_id = (uint64_t)blockIdx.x * 8 + threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    if (warp_id >= p.head_count * p.seq_len) return;
    const uint64_t head = warp_id / p.seq_len, query = warp_id % p.seq_len;
    const uint64_t kvh = head / p.group;
    uint64_t lo, hi;
    key_range(p, p.qpos0 + query, lo, hi);
    const float* qrow = p.q + query * p.q_model_dim + head * p.head_dim;
    float* orow = p.out + (query * p.head_count + head) * p.value_dim;
    for (uint64_t d = lane; d < p.value_dim; d += 32) orow[d] = 0.0f;
    float m = __int_as_float(0xff800000), l = 0.0f;
    for (uint64_t key = lo; key < hi; key++) {
        const float* krow = p.k + key * p.kv_model_dim + kvh * p.head_dim;
        float dot = 0.0f;
        for (uint64_t d = lane; d < p.head_dim; d += 32) dot += qrow[d] * krow[d];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        const float s = dot * p.scale;
        const float m_new = fmaxf(m, s);
        const float alpha = expf(m - m_new);
        const float e = expf(s - m_new);
        const float l_new = l * alpha + e;
        const float keep = (l * alpha) / l_new, w = e / l_new;
        const float* vrow = p.v + key * p.v_model_dim + kvh * p.value_dim;
        for (uint64_t d = lane; d < p.value_dim; d += 32) orow[d] = orow[d] * keep + w * vrow[d];
        m = m_new;
        l = l_new;
    }
}

// ---- short key spans: the whole span resident in shared memory ------------------------------
// When every CTA's admitted keys fit in shared memory (a short sequence, or a short window),
// the softmax needs no online merge: a CTA of 256 threads serves kShortQ queries of one head and
// copies the span of K and V once (cp.async); then each warp takes one query row on its own, with
// no further CTA-wide barrier:
//   1. scores: lane u takes keys u, u + 32, ... of the span (its K rows read as 16-byte chunks,
//      the query row held in registers or read as broadcasts);
//   2. the row's max, exp, sum and the weights divided by the sum, by warp shuffles -- the
//      reference's order (src/kernels.cu:1899-1958) -- masked keys weigh exactly 0;
//   3. P.V: lane u owns output columns D / 32 * u .. + D / 32 - 1; each key's weight comes from
//      the lane that holds it by a shuffle, its V row from shared memory.
// This launches one kernel with ceil(S / 8) * H CTAs and no split pass, so a decoder layer's
// attention (S = 128) is one short kernel instead of a tensor-core pipeline that would keep
// only H CTAs busy.
constexpr int kShortQ = 8;
constexpr int kShortThreads = 256;
static_assert(kShortThreads / 32 == kShortQ, "one warp per query row");

// Key capacity limit per head dimension (shared memory: about 400 B a key at D = 64).
template <int D>
constexpr uint32_t short_cap_limit() {
    return D <= 32 ? 512 : D <= 64 ? 384 : 192;
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Shared-memory plan for `cap` keys: K rows padded to D + 4 floats (an odd number of 16-byte
// chunks, so a lane per key reads conflict-free), V rows dense, then Q.
template <int D>
struct ShortPlan {
    static constexpr int kKStride = D + 4;
    __host__ __device__ static uint32_t off_v(uint32_t cap) { return cap * kKStride * 4; }
    __host__ __device__ static uint32_t off_q(uint32_t cap) { return off_v(cap) + cap * D * 4; }
    __host__ __device__ static uint32_t bytes(uint32_t cap) { return off_q(cap) + kShortQ * D * 4; }
};

template <int D>
__global__ void __launch_bounds__(kShortThreads) attention_short_kernel(AttnP p, uint32_t cap, int* error) {
    pdl_enter();
    using P = ShortPlan<D>;
    constexpr int kT = (int)(short_cap_limit<D>() / 32);  // keys per lane at most
    constexpr int C = D / 32;                              // output columns per lane
    constexpr bool kQRegs = D <= 64;                       // the query row in registers
    extern __shared__ __align__(16) unsigned char smem[];
    float* ks = reinterpret_cast<float*>(smem);
    float* vs = reinterpret_cast<float*>(smem + P::off_v(cap));
    float* qs = reinterpret_cast<float*>(smem + P::off_q(cap));
    const float ninf = __int_as_float(0xff800000);
    const uint64_t head = blockIdx.y, kvh = head / p.group;
    const uint64_t q0 = (uint64_t)blockIdx.x * kShortQ;
    const int nq = (int)min((uint64_t)kShortQ, p.seq_len - q0);
    uint64_t span_lo, span_hi, tmp;
    key_range(p, p.qpos0 + q0, span_lo, tmp);
    key_range(p, p.qpos0 + q0 + nq - 1, tmp, span_hi);
    if (span_lo > span_hi) span_lo = span_hi;
    const uint64_t span = span_hi - span_lo;
    if (span > cap) {  // the host sizes cap for the widest span; never taken
        if (threadIdx.x == 0) atomicExch(error, 1);
        return;
    }
    const int n = (int)span;
    constexpr int C4 = D / 4;  // 16-byte chunks per row

    for (int i = threadIdx.x; i < kShortQ * C4; i += kShortThreads) {
        const int qi = i / C4, c = i % C4;
        float* dst = qs + qi * D + c * 4;
        if (qi < nq) cp_async16(dst, p.q + (q0 + qi) * p.q_model_dim + head * D + c * 4);
        else *reinterpret_cast<float4*>(dst) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (int i = threadIdx.x; i < n * C4; i += kShortThreads) {
        const int j = i / C4, c = i % C4;
        const uint64_t key = span_lo + j;
        cp_async16(ks + j * P::kKStride + c * 4, p.k + key * p.kv_model_dim + kvh * D + c * 4);
        cp_async16(vs + j * D + c * 4, p.v + key * p.v_model_dim + kvh * D + c * 4);
    }
    cp_async_wait_all();
    __syncthreads();

    const int qi = threadIdx.x / 32, lane = threadIdx.x % 32;
    if (qi >= nq) return;
    uint64_t qlo, qhi;
    key_range(p, p.qpos0 + q0 + qi, qlo, qhi);
    const float* qrow = qs + qi * D;
    float4 qr[kQRegs ? C4 : 1];
    if constexpr (kQRegs) {
#pragma unroll
        for (int c = 0; c < C4; c++) qr[c] = reinterpret_cast<const float4*>(qrow)[c];
    }
    // 1. scores of this lane's keys (masked: -inf)
    float sc[kT];
    float m = ninf;
#pragma unroll
    for (int t = 0; t < kT; t++) {
        sc[t] = ninf;
        const int j = 32 * t + lane;
        if (32 * t >= n) continue;
        if (j < n) {
            const float4* kr = reinterpret_cast<const float4*>(ks + j * P::kKStride);
            float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // four independent chains over the columns
#pragma unroll
            for (int c = 0; c < C4; c++) {
                const float4 kk = kr[c];
                const float4 qq = kQRegs ? qr[kQRegs ? c : 0] : reinterpret_cast<const float4*>(qrow)[c];
                acc[c & 3] += qq.x * kk.x + qq.y * kk.y + qq.z * kk.z + qq.w * kk.w;
            }
            const uint64_t key = span_lo + j;
            sc[t] = (key >= qlo && key < qhi) ? ((acc[0] + acc[1]) + (acc[2] + acc[3])) * p.scale : ninf;
        }
        m = fmaxf(m, sc[t]);
    }
    // 2. softmax over the row: max, exp, sum by shuffles; weights e / sum
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.0f;
#pragma unroll
    for (int t = 0; t < kT; t++) {
        if (32 * t >= n) break;
        sc[t] = (m == ninf || sc[t] == ninf) ? 0.0f : expf(sc[t] - m);
        l += sc[t];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
#pragma unroll
    for (int t = 0; t < kT; t++) {
        if (32 * t >= n) break;
        sc[t] = m == ninf ? 0.0f : sc[t] / l;
    }
    // 3. P.V: columns C * lane .. C * lane + C - 1, keys in order, four chains
    float o[4][C];
#pragma unroll
    for (int e = 0; e < C; e++) o[0][e] = o[1][e] = o[2][e] = o[3][e] = 0.0f;
#pragma unroll
    for (int t = 0; t < kT; t++) {
        if (32 * t >= n) break;
        const int kn = min(32, n - 32 * t);
        const float* vrow0 = vs + (32 * t) * D + C * lane;
        int u = 0;
        for (; u + 3 < kn; u += 4) {
            float w[4];
#pragma unroll
            for (int h = 0; h < 4; h++) w[h] = __shfl_sync(0xffffffffu, sc[t], u + h);
            const float* v0 = vrow0 + u * D;
#pragma unroll
            for (int h = 0; h < 4; h++)
#pragma unroll
                for (int e = 0; e < C; e++) o[h][e] += w[h] * v0[h * D + e];
        }
        for (; u < kn; u++) {
            const float w0 = __shfl_sync(0xffffffffu, sc[t], u);
            const float* v0 = vrow0 + u * D;
#pragma unroll
            for (int e = 0; e < C; e++) o[0][e] += w0 * v0[e];
        }
    }
    float* orow = p.out + ((q0 + qi) * p.head_count + head) * D + C * lane;
#pragma unroll
    for (int e = 0; e < C; e++) orow[e] = (o[0][e] + o[1][e]) + (o[2][e] + o[3][e]);
}

// Largest key span any CTA of the short kernel sees: all keys, or a causal window plus the
// CTA's extra queries (a window implies causal masking).
uint64_t short_span_bound(const AttnP& p) {
    uint64_t span = p.kv_seq_len;
    if (p.window >= 0 && p.causal) span = std::min<uint64_t>(span, (uint64_t)p.window + kShortQ - 1);
    return span;
}

template <int D>
mg_status launch_short(Device* d, const AttnP& p, uint32_t cap) {
    using P = ShortPlan<D>;
    const uint32_t smem = P::bytes(cap);
    static uint32_t configured[64] = {0};
    if (configured[d->ordinal & 63] < smem) {
        MG_CUDA(cudaFuncSetAttribute(attention_short_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)ShortPlan<D>::bytes(short_cap_limit<D>())),
                "configuring the short attention kernel");
        configured[d->ordinal & 63] = ShortPlan<D>::bytes(short_cap_limit<D>());
    }
    dim3 grid((unsigned)((p.seq_len + kShortQ - 1) / kShortQ), (unsigned)p.head_count);
    enqueue(d, attention_short_kernel<D>, grid, kShortThreads, smem, p, cap, d->flags + 2);
    return launched(d, "short attention launch");
}

// ---- decode: one query row against a key history, keys split across CTAs -------------------
// The reference's attention_split / attention_combine (src/kernels.rs:6939-7078): chunks of
// keys scored by separate CTAs, merged in chunk order.  Here a CTA of 128 threads takes one
// head and 128 keys (a thread per key for the scores; a thread per output column for P.V, so
// V's rows are read coalesced) and writes its partial (max, sum, unnormalised output); the
// combine kernel rescales the partials to the common max and adds them in chunk order.  Bound
// by reading K and V once.  With a captured step's advancing key count the grid covers every
// row K and V hold and the admitted count is read at run time.
constexpr int kDecodeKeys = 128;
constexpr int kDecodeMaxDim = 256;

struct DecodeP {
    const float* q;
    const float* k;
    const float* v;
    float* partial;  // [head][chunk][value_dim + 2]: max, sum, output
    float* out;
    uint64_t kv_seq_len, head_count, group, head_dim, value_dim, q_model_dim, kv_model_dim, v_model_dim, chunks;
    int causal;
    int64_t window;
    float scale;
    const uint64_t* step;
    int vec;  // K rows 16-byte aligned: float4 loads
    int* error;
};

// Max (or sum) over the CTA's 128 threads of each of G values, one pair of barriers for all.
template <int G>
__device__ __forceinline__ void block_reduce_g(float (&v)[G], float (*red)[4], bool is_max) {
#pragma unroll
    for (int g = 0; g < G; g++)
        for (int o = 16; o > 0; o >>= 1) {
            const float w = __shfl_xor_sync(0xffffffffu, v[g], o);
            v[g] = is_max ? fmaxf(v[g], w) : v[g] + w;
        }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0)
#pragma unroll
        for (int g = 0; g < G; g++) red[g][warp] = v[g];
    __syncthreads();
#pragma unroll
    for (int g = 0; g < G; g++)
        v[g] = is_max ? fmaxf(fmaxf(red[g][0], red[g][1]), fmaxf(red[g][2], red[g][3]))
                      : (red[g][0] + red[g][1]) + (red[g][2] + red[g][3]);
}

// G > 1: a CTA takes the G query heads of one KV head (blockIdx.y = KV head), so K and V are
// read once for the group (the reference's grouped decode kernel); G == 1: blockIdx.y = the
// query head.  blockIdx.x = the chunk of keys.
template <int G>
__global__ void __launch_bounds__(kDecodeKeys) attention_decode_kernel(DecodeP p) {
    pdl_enter();
    __shared__ float qs[G][kDecodeMaxDim];
    __shared__ float ps[G][kDecodeKeys];
    __shared__ float red[G][4];
    const uint64_t h0 = G == 1 ? blockIdx.y : (uint64_t)blockIdx.y * G;
    const uint64_t kvh = G == 1 ? blockIdx.y / p.group : blockIdx.y;
    const uint64_t c = blockIdx.x;
    const uint64_t n_keys = p.kv_seq_len + (p.step ? *p.step : 0);
    const uint64_t qpos = n_keys - 1;  // the row's position: the last admitted key
    uint64_t lo = 0;
    if (p.window >= 0) {
        const uint64_t back = (uint64_t)p.window - 1;
        lo = qpos > back ? qpos - back : 0;
    }
#pragma unroll
    for (int g = 0; g < G; g++)
        for (uint64_t d = threadIdx.x; d < p.head_dim; d += kDecodeKeys) qs[g][d] = p.q[(h0 + g) * p.head_dim + d];
    __syncthreads();
    const uint64_t key = c * kDecodeKeys + threadIdx.x;
    const bool live = key >= lo && key < n_keys;
    float s[G];
#pragma unroll
    for (int g = 0; g < G; g++) s[g] = __int_as_float(0xff800000);
    if (live) {
        const float* kr = p.k + key * p.kv_model_dim + kvh * p.head_dim;
        float dot[G];
#pragma unroll
        for (int g = 0; g < G; g++) dot[g] = 0.0f;
        if (p.vec) {  // the same sums, in the same order, from 16-byte loads
            for (uint64_t d = 0; d < p.head_dim; d += 4) {
                const float4 kv = *reinterpret_cast<const float4*>(kr + d);
#pragma unroll
                for (int g = 0; g < G; g++) {
                    dot[g] += qs[g][d] * kv.x;
                    dot[g] += qs[g][d + 1] * kv.y;
                    dot[g] += qs[g][d + 2] * kv.z;
                    dot[g] += qs[g][d + 3] * kv.w;
                }
            }
        } else {
            for (uint64_t d = 0; d < p.head_dim; d++) {
                const float kv = kr[d];
#pragma unroll
                for (int g = 0; g < G; g++) dot[g] += qs[g][d] * kv;
            }
        }
#pragma unroll
        for (int g = 0; g < G; g++) s[g] = dot[g] * p.scale;
    }
    float m[G];
#pragma unroll
    for (int g = 0; g < G; g++) m[g] = s[g];
    block_reduce_g<G>(m, red, true);
    if (m[0] == __int_as_float(0xff800000)) {  // no admitted key in this chunk (for any head)
        if (threadIdx.x == 0)
#pragma unroll
            for (int g = 0; g < G; g++) {
                float* part = p.partial + ((h0 + g) * p.chunks + c) * (p.value_dim + 2);
                part[0] = __int_as_float(0xff800000);
                part[1] = 0.0f;
            }
        return;
    }
    float l[G];
#pragma unroll
    for (int g = 0; g < G; g++) {
        l[g] = live ? expf(s[g] - m[g]) : 0.0f;
        ps[g][threadIdx.x] = l[g];
    }
    block_reduce_g<G>(l, red, false);  // its barriers also publish ps
    const uint64_t k0 = c * kDecodeKeys;
    const int nk = (int)min((uint64_t)kDecodeKeys, n_keys - k0);
    for (uint64_t d = threadIdx.x; d < p.value_dim; d += kDecodeKeys) {
        const float* vc = p.v + k0 * p.v_model_dim + kvh * p.value_dim + d;
        float acc[G];
#pragma unroll
        for (int g = 0; g < G; g++) acc[g] = 0.0f;
        for (int j = 0; j < nk; j++) {
            const float vv = vc[(uint64_t)j * p.v_model_dim];
#pragma unroll
            for (int g = 0; g < G; g++) acc[g] += ps[g][j] * vv;
        }
#pragma unroll
        for (int g = 0; g < G; g++) p.partial[((h0 + g) * p.chunks + c) * (p.value_dim + 2) + 2 + d] = acc[g];
    }
    if (threadIdx.x == 0)
#pragma unroll
        for (int g = 0; g < G; g++) {
            float* part = p.partial + ((h0 + g) * p.chunks + c) * (p.value_dim + 2);
            part[0] = m[g];
            part[1] = l[g];
        }
}

// The TMA form (16-byte aligned rows, head dimensions multiples of 4): a CTA of 256 threads
// takes a span of keys of one KV head (about three CTAs per SM over the grid) and its G query
// heads, and streams the span in tiles of 32 keys through a 2-stage ring of TMA copies ([32][D]
// of K and [32][Dv] of V per stage).  Each warp takes 4 keys of every tile and keeps its own
// online softmax (running max, sum and unnormalised output) over them: scores with 8 lanes per
// key (16-byte column chunks, a 3-level butterfly per head), max and sum by shuffles inside the
// warp, P.V with each lane owning output columns 4 lane .. 4 lane + 3 (and + 128) read as
// 16-byte loads of the V rows -- no CTA-wide barrier per tile but the one that frees a stage.
// The warps' states are merged once, in warp order, into the span's partial (max, sum,
// output) for the combine kernel.
constexpr int kDecodeThreads = 256;
constexpr int kDecodeStages = 3;  // 2 -> 3: 0.0567 -> 0.0560 ms at 32768 keys
constexpr int kDecodeTileKeys = 32;  // 4 keys per warp
constexpr int kDecodeStageBytes = kDecodeTileKeys * 2 * kDecodeMaxDim * 4;  // 64 KB at D = Dv = 256

template <int G, int C>  // C: 128-column chunks of the output (Dv <= 128 * C)
__device__ __forceinline__ void decode_tma_span(const CUtensorMap& map_k, const CUtensorMap& map_v, const DecodeP& p,
                                                uint64_t span) {
    using namespace sm100;
    constexpr int kc = kDecodeTileKeys;
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(16) float qs[G][kDecodeMaxDim];
    __shared__ float wm[8][G], wl[8][G];
    __shared__ uint64_t bars[kDecodeStages], empty[kDecodeStages];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 127u) & ~127u;
    float* smem_f = reinterpret_cast<float*>(smem_raw + (base - raw));
    const uint64_t h0 = G == 1 ? blockIdx.y : (uint64_t)blockIdx.y * G;
    const uint64_t kvh = G == 1 ? blockIdx.y / p.group : blockIdx.y;
    const uint64_t c = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint64_t D = p.head_dim, DV = p.value_dim;
    const uint32_t D32 = (uint32_t)D, DV32 = (uint32_t)DV;  // shared-memory offsets stay 32-bit
    const uint32_t k_bytes = (uint32_t)(4 * kc * D);
    const uint32_t stage_bytes = (uint32_t)(4 * kc * (D + DV));
    pdl_enter();  // K and V may have just been written (kv-write)
    const uint64_t n_keys = p.kv_seq_len + (p.step ? *p.step : 0);
    const uint64_t qpos = n_keys - 1;
    uint64_t lo = 0;
    if (p.window >= 0) {
        const uint64_t back = (uint64_t)p.window - 1;
        lo = qpos > back ? qpos - back : 0;
    }
    // This CTA's tiles: from the span's start (or the first tile holding `lo`) to its admitted end.
    const uint64_t k_begin = c * span, k_end = min(k_begin + span, n_keys);
    const uint64_t first = lo > k_begin ? k_begin + (lo - k_begin) / kc * kc : k_begin;
    const int tiles = k_end > first ? (int)((k_end - first + kc - 1) / kc) : 0;
    const uint64_t pstride = p.chunks * (DV + 2);
    float* part0 = p.partial + (h0 * p.chunks + c) * (DV + 2);
    const float kNegInf = __int_as_float(0xff800000);
    if (tiles == 0) {  // no admitted key here: an empty partial, no copies
        if (threadIdx.x == 0)
            for (int g = 0; g < G; g++) {
                part0[g * pstride] = kNegInf;
                part0[g * pstride + 1] = 0.0f;
            }
        return;
    }
    auto issue = [&](int t) {
        const int st = t % kDecodeStages;
        const uint32_t dst = base + (uint32_t)st * stage_bytes;
        const int key = (int)(first + (uint64_t)t * kc);
        mbar_arrive_expect_tx(smem_u32(&bars[st]), stage_bytes);
        tma_load_2d(dst, &map_k, smem_u32(&bars[st]), (int)(kvh * D), key);
        tma_load_2d(dst + k_bytes, &map_v, smem_u32(&bars[st]), (int)(kvh * DV), key);
    };
    if (threadIdx.x == 0) {
        for (int st = 0; st < kDecodeStages; st++) {
            mbar_init(smem_u32(&bars[st]), 1);
            mbar_init(smem_u32(&empty[st]), kDecodeThreads / 32);  // every warp leaves the stage
        }
        fence_barrier_init();
        for (int t = 0; t < min(tiles, kDecodeStages); t++) issue(t);
    }
#pragma unroll
    for (int g = 0; g < G; g++)
        for (uint64_t d = threadIdx.x; d < D; d += kDecodeThreads) qs[g][d] = p.q[(h0 + g) * D + d];
    __syncthreads();  // the barriers' initialisation and q are visible
    const int sk = lane >> 3, sc4 = (lane & 7) * 4;  // scores: key sk of the warp's 4, columns sc4 + 32 i
    // Up to 4 query heads with head dimensions up to 128 (C = 1 is launched only then): this
    // lane's 16 query columns per head stay in registers for the whole span instead of being
    // re-read from shared memory per key.
    constexpr bool kQRegs = C == 1 && G <= 4;
    uint64_t q2[kQRegs ? G : 1][kQRegs ? 8 : 1];  // column pairs (sc4 + 32 i + 2 h, + 1), slot 2 i + h
    if constexpr (kQRegs) {
#pragma unroll
        for (int g = 0; g < G; g++)
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const uint64_t d = sc4 + 32 * i;
                const float4 qv = d < D ? *reinterpret_cast<const float4*>(&qs[g][d]) : make_float4(0.f, 0.f, 0.f, 0.f);
                q2[g][2 * i] = f2(qv.x, qv.y);
                q2[g][2 * i + 1] = f2(qv.z, qv.w);
            }
    }
    // P.V: this lane's output columns 4 lane + 128 i + e as packed pairs, slot 2 i + e / 2
    float m[G], l[G];
    uint64_t acc2[G][2 * C];
#pragma unroll
    for (int g = 0; g < G; g++) {
        m[g] = kNegInf;
        l[g] = 0.0f;
#pragma unroll
        for (int e = 0; e < 2 * C; e++) acc2[g][e] = 0ull;
    }
    bool ok = true;
    for (int t = 0; t < tiles; t++) {
        const int st = t % kDecodeStages;
        if (!mbar_wait(smem_u32(&bars[st]), (uint32_t)(t / kDecodeStages) & 1u)) ok = false;
        if (!__all_sync(0xffffffffu, ok)) {  // warps run ahead of one another: no CTA barrier per tile
            ok = false;
            if (lane == 0) atomicExch(p.error, 1);
            break;
        }
        const float* ks = smem_f + (uint64_t)st * (stage_bytes / 4);
        const float* vs = ks + (uint64_t)kc * D;
        const int jb = warp * 4, j = jb + sk;
        float sc[G];
#pragma unroll
        for (int g = 0; g < G; g++) sc[g] = 0.0f;
        if constexpr (kQRegs) {
            uint64_t s2[G];  // even and odd columns, one lane each
#pragma unroll
            for (int g = 0; g < G; g++) s2[g] = 0ull;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const uint32_t d = (uint32_t)sc4 + 32u * i;
                if (d >= D32) break;
                const float4 kv = *reinterpret_cast<const float4*>(ks + (uint32_t)j * D32 + d);
                const uint64_t k01 = f2(kv.x, kv.y), k23 = f2(kv.z, kv.w);
#pragma unroll
                for (int g = 0; g < G; g++) {
                    f2fma(s2[g], q2[g][2 * i], k01);
                    f2fma(s2[g], q2[g][2 * i + 1], k23);
                }
            }
#pragma unroll
            for (int g = 0; g < G; g++) {
                const float2 sv = f2split(s2[g]);
                sc[g] = sv.x + sv.y;
            }
        } else {
            for (uint64_t d = sc4; d < D; d += 32) {
                const float4 kv = *reinterpret_cast<const float4*>(ks + (uint64_t)j * D + d);
#pragma unroll
                for (int g = 0; g < G; g++) {
                    const float4 qv = *reinterpret_cast<const float4*>(&qs[g][d]);
                    sc[g] += qv.x * kv.x + qv.y * kv.y + qv.z * kv.z + qv.w * kv.w;
                }
            }
        }
        const uint64_t key = first + (uint64_t)t * kc + j;
        const bool live = key >= lo && key < k_end;
        float pk[G][4];  // the weights of the warp's 4 keys, the same in every lane
#pragma unroll
        for (int g = 0; g < G; g++) {
            for (int o = 4; o > 0; o >>= 1) sc[g] += __shfl_xor_sync(0xffffffffu, sc[g], o);
            sc[g] = live ? sc[g] * p.scale : kNegInf;
            float tmx = fmaxf(sc[g], __shfl_xor_sync(0xffffffffu, sc[g], 8));
            tmx = fmaxf(tmx, __shfl_xor_sync(0xffffffffu, tmx, 16));
            // The reference max moves only when a tile's max passes it by more than e^8 (the
            // weights then stay <= e^8, safe in f32, and the sums and outputs are rescaled only
            // then); tmx and m are the same in every lane, so the branch is warp-uniform.
            if (m[g] == kNegInf || tmx > m[g] + 8.0f) {
                const float m_new = fmaxf(m[g], tmx);
                const float alpha = m[g] == kNegInf ? 0.0f : __expf(m[g] - m_new);
                m[g] = m_new;
                l[g] *= alpha;
                const uint64_t alpha2 = f2(alpha, alpha);
#pragma unroll
                for (int e = 0; e < 2 * C; e++) acc2[g][e] = f2mul(acc2[g][e], alpha2);
            }
            const float ex = (sc[g] != kNegInf && m[g] != kNegInf) ? __expf(sc[g] - m[g]) : 0.0f;
            float es = ex + __shfl_xor_sync(0xffffffffu, ex, 8);
            es += __shfl_xor_sync(0xffffffffu, es, 16);
            l[g] += es;
#pragma unroll
            for (int k = 0; k < 4; k++) pk[g][k] = __shfl_sync(0xffffffffu, ex, k * 8);
        }
#pragma unroll
        for (int i = 0; i < C; i++) {
            const uint32_t d = 4u * lane + 128u * i;
            if (d >= DV32) break;
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const float4 vv = *reinterpret_cast<const float4*>(vs + (uint32_t)(jb + k) * DV32 + d);
                const uint64_t v01 = f2(vv.x, vv.y), v23 = f2(vv.z, vv.w);
#pragma unroll
                for (int g = 0; g < G; g++) {
                    const uint64_t pp = f2(pk[g][k], pk[g][k]);
                    f2fma(acc2[g][2 * i], pp, v01);
                    f2fma(acc2[g][2 * i + 1], pp, v23);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&empty[st]));  // this warp is done with the stage
        if (threadIdx.x == 0 && t + kDecodeStages < tiles) {
            // the stage refills once every warp has left it
            if (mbar_wait(smem_u32(&empty[st]), (uint32_t)(t / kDecodeStages) & 1u)) {
                issue(t + kDecodeStages);
            } else {
                ok = false;  // the other warps' waits for this tile run out in turn
                atomicExch(p.error, 1);
            }
        }
    }
    ok = __syncthreads_and(ok) != 0;
    if (!ok) {  // give the copies in flight a second bound before the CTA exits
        if (threadIdx.x == 0)
            for (int st = 0; st < min(tiles, kDecodeStages); st++) (void)mbar_wait(smem_u32(&bars[st]), 0);
        __syncthreads();
        return;
    }
    // ---- merge the 8 warps' states (in warp order) into the span's partial -------------------
    if (lane == 0)
#pragma unroll
        for (int g = 0; g < G; g++) {
            wm[warp][g] = m[g];
            wl[warp][g] = l[g];
        }
    __syncthreads();
    float* wo = smem_f;  // [8][G][DV], the drained ring
#pragma unroll
    for (int g = 0; g < G; g++) {
        float mx = kNegInf;
        for (int w = 0; w < 8; w++) mx = fmaxf(mx, wm[w][g]);
        const float sc = m[g] == kNegInf ? 0.0f : expf(m[g] - mx);
#pragma unroll
        for (int i = 0; i < C; i++) {
            const uint64_t d = 4 * (uint64_t)lane + 128 * (uint64_t)i;
            if (d >= DV) break;
            const float2 a01 = f2split(acc2[g][2 * i]), a23 = f2split(acc2[g][2 * i + 1]);
            *reinterpret_cast<float4*>(wo + ((uint64_t)warp * G + g) * DV + d) =
                make_float4(a01.x * sc, a01.y * sc, a23.x * sc, a23.y * sc);
        }
    }
    __syncthreads();
    for (uint64_t e = threadIdx.x; e < (uint64_t)G * DV; e += kDecodeThreads) {
        const uint64_t g = e / DV, d = e % DV;
        float o = 0.0f;
        for (int w = 0; w < 8; w++) o += wo[((uint64_t)w * G + g) * DV + d];
        part0[g * pstride + 2 + d] = o;
    }
    if (threadIdx.x < G) {
        const int g = threadIdx.x;
        float mx = kNegInf;
        for (int w = 0; w < 8; w++) mx = fmaxf(mx, wm[w][g]);
        float ls = 0.0f;
        for (int w = 0; w < 8; w++)
            if (wm[w][g] != kNegInf) ls += wl[w][g] * expf(wm[w][g] - mx);
        part0[g * pstride] = mx;
        part0[g * pstride + 1] = ls;
    }
}

// The spans' partials of one query head merged (src/kernels.cu:2301-2800, attention_combine):
// the common max over the spans, each span's weight exp(m - max) (kept in `wts` for up to
// `cache` spans), the weighted sum of the span sums, and the output columns as the weighted
// sums of the span outputs in span order, eight spans' loads in flight per step.  T threads;
// `red` holds T / 32 floats.  Partials are read through the L2 (another CTA may have written
// them in this launch).
template <int T>
__device__ void combine_head(const DecodeP& p, uint64_t h, float* wts, uint64_t cache, float* red) {
    const uint64_t stride = p.value_dim + 2;
    const float* base = p.partial + h * p.chunks * stride;
    const float kNegInf = __int_as_float(0xff800000);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    auto block_max = [&](float v) {
        for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (lane == 0) red[warp] = v;
        __syncthreads();
        float r = red[0];
        for (int w = 1; w < T / 32; w++) r = fmaxf(r, red[w]);
        __syncthreads();
        return r;
    };
    auto block_sum = [&](float v) {  // a fixed order: lanes by butterfly, then warps in order
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) red[warp] = v;
        __syncthreads();
        float r = red[0];
        for (int w = 1; w < T / 32; w++) r += red[w];
        __syncthreads();
        return r;
    };
    float mx = kNegInf;
    for (uint64_t c = threadIdx.x; c < p.chunks; c += T) mx = fmaxf(mx, __ldcg(base + c * stride));
    mx = block_max(mx);
    const bool cached = p.chunks <= cache;
    float ls = 0.0f;
    for (uint64_t c = threadIdx.x; c < p.chunks; c += T) {
        const float mc = __ldcg(base + c * stride);
        const float w = mc != kNegInf ? expf(mc - mx) : 0.0f;
        if (cached) wts[c] = w;
        ls += __ldcg(base + c * stride + 1) * w;
    }
    const float l = block_sum(ls);  // its barriers also publish wts
    const float inv = l > 0.0f ? 1.0f / l : 0.0f;
    for (uint64_t d = threadIdx.x; d < p.value_dim; d += T) {
        const float* col = base + 2 + d;
        float o = 0.0f;
        for (uint64_t c0 = 0; c0 < p.chunks; c0 += 8) {
            float v[8], w[8];
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const uint64_t c = c0 + u;
                v[u] = c < p.chunks ? __ldcg(col + c * stride) : 0.0f;
                if (cached) {
                    w[u] = c < p.chunks ? wts[c] : 0.0f;
                } else {
                    const float mc = c < p.chunks ? __ldcg(base + c * stride) : kNegInf;
                    w[u] = mc != kNegInf ? expf(mc - mx) : 0.0f;
                }
            }
#pragma unroll
            for (int u = 0; u < 8; u++)
                if (c0 + u < p.chunks) o += v[u] * w[u];
        }
        p.out[h * p.value_dim + d] = o * inv;
    }
    __syncthreads();  // wts and red are reused by the next head
}

// One span of keys of one KV head set; attention_combine_kernel merges the spans.  (Merging in
// the set's last CTA instead, one launch, measured slower: 0.057 -> 0.068 ms at 32768 keys with
// that CTA combining its G heads one after another, 0.056 -> 0.060 ms with all its threads
// spread over the G heads' columns: the merge then runs after the slowest span's CTA, on one SM
// per head set, while the combine kernel is already resident and spreads the heads over CTAs.)
template <int G, int C>
__global__ void __launch_bounds__(kDecodeThreads) attention_decode_tma_kernel(const __grid_constant__ CUtensorMap map_k,
                                                                             const __grid_constant__ CUtensorMap map_v,
                                                                             DecodeP p, uint64_t span) {
    decode_tma_span<G, C>(map_k, map_v, p, span);
}

PFN_cuTensorMapEncodeTiled_v12000 decode_encode_fn() {
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

// Row-major [rows, cols] f32, box [box_rows, box_cols], no swizzle; rows past the end read as zero.
mg_status decode_map(CUtensorMap* map, const float* ptr, uint64_t rows, uint64_t cols, uint32_t box_cols,
                     uint32_t box_rows) {
    auto fn = decode_encode_fn();
    if (!fn) return fail(MG_DRIVER_FAILED, "the driver does not provide cuTensorMapEncodeTiled");
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols * sizeof(float)};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ptr), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(MG_DRIVER_FAILED, "encoding a TMA descriptor failed (CUresult %d)", (int)r);
    return MG_OK;
}

inline int decode_tma_smem(int g, uint64_t d, uint64_t dv) {
    const uint64_t ring = (uint64_t)kDecodeStages * kDecodeTileKeys * 4 * (d + dv);
    const uint64_t merge = 8ull * g * 4 * dv;  // the warps' outputs, in the drained ring
    return 128 + (int)(ring > merge ? ring : merge);
}

// Resident CTAs per SM of the G-head form at this shared-memory size (queried once per size).
template <int G, int C>
int decode_tma_occupancy(Device* d, int smem) {
    static int cached[64][4] = {{0}};
    static int cached_smem[64][4] = {{0}};
    const int slot = G == 1 ? 0 : G == 2 ? 1 : G == 4 ? 2 : 3;
    int& c = cached[d->ordinal & 63][slot];
    if (c == 0 || cached_smem[d->ordinal & 63][slot] != smem) {
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, attention_decode_tma_kernel<G, C>, kDecodeThreads, smem) !=
                cudaSuccess ||
            n < 1) {
            (void)cudaGetLastError();
            n = 1;
        }
        c = n;
        cached_smem[d->ordinal & 63][slot] = smem;
    }
    return c;
}

template <int G, int C>
mg_status launch_decode_tma(Device* d, const DecodeP& p, const CUtensorMap* maps, uint64_t span, dim3 grid) {
    const int smem = decode_tma_smem(G, p.head_dim, p.value_dim);
    enqueue(d, attention_decode_tma_kernel<G, C>, grid, kDecodeThreads, (size_t)smem, maps[0], maps[1], p, span);
    return launched(d, "decode attention launch");
}

template <int G, int C>
mg_status configure_decode_tma(Device* d) {
    static bool configured[64] = {false};
    if (!configured[d->ordinal & 63]) {
        MG_CUDA(cudaFuncSetAttribute(attention_decode_tma_kernel<G, C>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     128 + kDecodeStages * kDecodeStageBytes),
                "configuring the decode attention kernel");
        configured[d->ordinal & 63] = true;
    }
    return MG_OK;
}

// The spans' partials of one query head merged (src/kernels.cu:2301-2800, attention_combine):
// the common max over the spans, each span's weight exp(m - max) (kept in shared memory for up
// to kCombineWeights spans), the weighted sum of the span sums, and the output columns as the
// weighted sums of the span outputs in span order, eight spans' loads in flight per step.
constexpr int kCombineWeights = 2048;

__global__ void __launch_bounds__(kDecodeKeys) attention_combine_kernel(DecodeP p) {
    pdl_enter();
    __shared__ float wts[kCombineWeights];
    __shared__ float red[kDecodeKeys / 32];
    combine_head<kDecodeKeys>(p, blockIdx.x, wts, kCombineWeights, red);
}

mg_status attention_decode(Device* d, const k::AttentionArgs& a) {
    DecodeP p;
    p.q = a.q;
    p.k = a.k;
    p.v = a.v;
    p.out = a.out;
    p.kv_seq_len = a.kv_seq_len;
    p.head_count = a.head_count;
    p.group = a.head_count / a.kv_head_count;
    p.head_dim = a.head_dim;
    p.value_dim = a.value_dim;
    p.q_model_dim = a.q_model_dim;
    p.kv_model_dim = a.kv_model_dim;
    p.v_model_dim = a.v_model_dim;
    p.causal = a.causal;
    p.window = a.window;
    p.scale = a.scale;
    p.step = a.step;
    p.vec = (reinterpret_cast<uintptr_t>(a.k) & 15) == 0 && a.kv_model_dim % 4 == 0 && a.head_dim % 4 == 0;
    p.error = d->flags + 2;
    const uint64_t keys = a.step ? a.kv_rows : a.kv_seq_len;  // the grid covers what may be admitted
    auto al16 = [](const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15) == 0; };
    const bool tma = al16(a.k) && al16(a.v) && a.head_dim % 4 == 0 && a.value_dim % 4 == 0 &&
                     a.kv_model_dim % 4 == 0 && a.v_model_dim % 4 == 0 && a.kv_rows < (1ull << 31) &&
                     a.kv_model_dim < (1ull << 31) && a.v_model_dim < (1ull << 31);
    const int kc = tma ? kDecodeTileKeys : kDecodeKeys;
    // TMA form: spans of whole tiles, one wave of CTAs (as many per SM as fit).
    uint64_t span = (uint64_t)kc;
    if (tma) {
        const int G = (p.group == 2 || p.group == 4 || p.group == 8) ? (int)p.group : 1;
        const int smem = decode_tma_smem(G, a.head_dim, a.value_dim);
        int per_sm = 1;
        const bool wide = a.value_dim > 128 || a.head_dim > 128;  // C = 2 (C = 1 holds q in registers)
#define MG_DECODE_OCC(GG)                                                              \
    if (wide) {                                                                        \
        MG_TRY((configure_decode_tma<GG, 2>(d)));                                      \
        per_sm = decode_tma_occupancy<GG, 2>(d, smem);                                 \
    } else {                                                                           \
        MG_TRY((configure_decode_tma<GG, 1>(d)));                                      \
        per_sm = decode_tma_occupancy<GG, 1>(d, smem);                                 \
    }
        switch (G) {
            case 2: MG_DECODE_OCC(2) break;
            case 4: MG_DECODE_OCC(4) break;
            case 8: MG_DECODE_OCC(8) break;
            default: MG_DECODE_OCC(1) break;
        }
#undef MG_DECODE_OCC
        const uint64_t sets = G == 1 ? a.head_count : a.kv_head_count;  // CTAs per span of keys
        const uint64_t want = std::max<uint64_t>(1, (uint64_t)per_sm * d->sm_count / std::max<uint64_t>(1, sets));
        span = std::max<uint64_t>(1, (keys + want - 1) / want);
        span = (span + kc - 1) / kc * kc;
    }
    p.chunks = std::max<uint64_t>(1, (keys + span - 1) / span);
    if (p.chunks > 0x7FFFFFFFull) return fail(MG_SHAPE_UNSUPPORTED, "attention has too many keys for the decode grid");
    MG_TRY(scratch(d, 6, a.head_count * p.chunks * (a.value_dim + 2) * sizeof(float), (void**)&p.partial));
    const dim3 by_kv((unsigned)p.chunks, (unsigned)a.kv_head_count), by_q((unsigned)p.chunks, (unsigned)a.head_count);
    if (tma) {
        CUtensorMap maps[2];
        MG_TRY(decode_map(&maps[0], a.k, a.kv_rows, a.kv_model_dim, (uint32_t)a.head_dim, (uint32_t)kc));
        MG_TRY(decode_map(&maps[1], a.v, a.kv_rows, a.v_model_dim, (uint32_t)a.value_dim, (uint32_t)kc));
        const bool wide = a.value_dim > 128 || a.head_dim > 128;  // C = 2 (C = 1 holds q in registers)
        mg_status ls = MG_OK;
        switch (p.group) {
            case 2: ls = wide ? launch_decode_tma<2, 2>(d, p, maps, span, by_kv) : launch_decode_tma<2, 1>(d, p, maps, span, by_kv); break;
            case 4: ls = wide ? launch_decode_tma<4, 2>(d, p, maps, span, by_kv) : launch_decode_tma<4, 1>(d, p, maps, span, by_kv); break;
            case 8: ls = wide ? launch_decode_tma<8, 2>(d, p, maps, span, by_kv) : launch_decode_tma<8, 1>(d, p, maps, span, by_kv); break;
            default: ls = wide ? launch_decode_tma<1, 2>(d, p, maps, span, by_q) : launch_decode_tma<1, 1>(d, p, maps, span, by_q); break;
        }
        MG_TRY(ls);
        enqueue(d, attention_combine_kernel, dim3((unsigned)a.head_count), kDecodeKeys, 0, p);
        return launched(d, "decode attention combine launch");
    }
    switch (p.group) {
        case 2: enqueue(d, attention_decode_kernel<2>, by_kv, kDecodeKeys, 0, p); break;
        case 4: enqueue(d, attention_decode_kernel<4>, by_kv, kDecodeKeys, 0, p); break;
        case 8: enqueue(d, attention_decode_kernel<8>, by_kv, kDecodeKeys, 0, p); break;
        default: enqueue(d, attention_decode_kernel<1>, by_q, kDecodeKeys, 0, p); break;
    }
    MG_TRY(launched(d, "decode attention launch"));
    enqueue(d, attention_combine_kernel, dim3((unsigned)a.head_count), kDecodeKeys, 0, p);
    return launched(d, "decode attention combine launch");
}

}  // namespace

namespace k {

bool attention_tc_eligible(const AttentionArgs& a);
mg_status attention_tc(Device* d, const AttentionArgs& a);

mg_status attention(Device* d, const AttentionArgs& a) {
    if (a.seq_len == 0 || a.head_count == 0) return MG_OK;
    AttnP p;
    p.q = a.q;
    p.k = a.k;
    p.v = a.v;
    p.out = a.out;
    p.seq_len = a.seq_len;
    p.kv_seq_len = a.kv_seq_len;
    p.head_count = a.head_count;
    p.group = a.head_count / a.kv_head_count;
    p.head_dim = a.head_dim;
    p.value_dim = a.value_dim;
    p.q_model_dim = a.q_model_dim;
    p.kv_model_dim = a.kv_model_dim;
    p.v_model_dim = a.v_model_dim;
    p.causal = a.causal;
    p.window = a.window;
    p.qpos0 = a.query_position_offset;
    p.scale = a.scale;
    const bool aligned = ((reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.k) |
                           reinterpret_cast<uintptr_t>(a.v) | reinterpret_cast<uintptr_t>(a.out)) & 15) == 0 &&
                         a.q_model_dim % 4 == 0 && a.kv_model_dim % 4 == 0 && a.v_model_dim % 4 == 0;
    if (a.head_count > 65535) return fail(MG_SHAPE_UNSUPPORTED, "attention head_count exceeds the launch grid");
    // One query row (a decode step): keys split across CTAs.
    const bool decode = a.seq_len == 1 && a.head_dim <= kDecodeMaxDim && a.value_dim <= kDecodeMaxDim;
    if (decode) return attention_decode(d, a);
    if (a.step)
        return fail(MG_CAPTURE_UNSUPPORTED,
                    "an advancing key_count needs a single query row with head and value dimensions of at most %d",
                    kDecodeMaxDim);
    // Short spans: one short kernel when every CTA's keys fit in shared memory and the grid is
    // at most two waves; otherwise the tensor-core pipeline.
    if (aligned && a.value_dim == a.head_dim && (a.head_dim == 32 || a.head_dim == 64 || a.head_dim == 128)) {
        const uint64_t span = short_span_bound(p);
        const uint32_t limit = a.head_dim == 32 ? short_cap_limit<32>() : a.head_dim == 64 ? short_cap_limit<64>()
                                                                                            : short_cap_limit<128>();
        if (span <= limit) {
            const uint32_t cap = (uint32_t)std::min<uint64_t>(((span + 31) / 32) * 32, limit);
            const uint32_t smem = a.head_dim == 32 ? ShortPlan<32>::bytes(cap) : a.head_dim == 64 ? ShortPlan<64>::bytes(cap)
                                                                                                : ShortPlan<128>::bytes(cap);
            const uint64_t per_sm = std::max<uint64_t>(1, std::min<uint64_t>(8, (228ull * 1024) / (smem + 1024)));
            const uint64_t ctas = (a.seq_len + kShortQ - 1) / kShortQ * a.head_count;
            if (ctas <= 2 * per_sm * (uint64_t)d->sm_count) {
                if (a.head_dim == 32) return launch_short<32>(d, p, cap);
                if (a.head_dim == 64) return launch_short<64>(d, p, cap);
                return launch_short<128>(d, p, cap);
            }
        }
    }
    if (attention_tc_eligible(a)) return attention_tc(d, a);
    const bool tiled = aligned && a.value_dim == a.head_dim && (a.head_dim == 64 || a.head_dim == 128 ||
                                                                 a.head_dim == 32 || a.head_dim == 16);
    if (tiled) {
        dim3 grid((unsigned)((a.seq_len + BQ - 1) / BQ), (unsigned)a.head_count);
        switch (a.head_dim) {
            case 16: enqueue(d, attention_tile_kernel<1>, grid, kAttnThreads, 0, p); break;
            case 32: enqueue(d, attention_tile_kernel<2>, grid, kAttnThreads, 0, p); break;
            case 64: enqueue(d, attention_tile_kernel<4>, grid, kAttnThreads, 0, p); break;
            default: enqueue(d, attention_tile_kernel<8>, grid, kAttnThreads, 0, p); break;
        }
        return launched(d, "attention kernel launch");
    }
    const uint64_t warps = a.head_count * a.seq_len;
    const uint64_t blocks = (warps + 7) / 8;
    if (blocks > 0x7FFFFFFFull) return fail(MG_SHAPE_UNSUPPORTED, "attention launch size overflows");
    enqueue(d, attention_generic_kernel, (unsigned)blocks, 256, 0, p);
    return launched(d, "attention kernel launch");
}

}  // namespace k
}  // namespace mg
