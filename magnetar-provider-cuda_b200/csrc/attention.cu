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
#include "internal.h"

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
// the softmax needs no online merge: a CTA of 256 threads serves kShortQ queries of one head,
// copies the span of K and V once (cp.async), then
//   1. scores: one thread per key, kShortQ dot products against the broadcast Q rows;
//   2. one warp per query row: max, exp, sum, and the weights divided by the sum -- the
//      reference's order (src/kernels.cu:1899-1958) -- masked keys weigh exactly 0;
//   3. P.V: one thread per output column and kShortQ * D / 256 queries.
// This launches one kernel with ceil(S / 8) * H CTAs and no split pass, so a decoder layer's
// attention (S = 128) is one short kernel instead of a tensor-core pipeline that would keep
// only H CTAs busy.
constexpr int kShortQ = 8;
constexpr int kShortThreads = 256;

// Key capacity limit per head dimension (shared memory: about 560 B a key at D = 64).
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
// chunks, so one thread per key reads conflict-free), V rows dense, Q, and P [kShortQ][cap].
template <int D>
struct ShortPlan {
    static constexpr int kKStride = D + 4;
    __host__ __device__ static uint32_t off_v(uint32_t cap) { return cap * kKStride * 4; }
    __host__ __device__ static uint32_t off_q(uint32_t cap) { return off_v(cap) + cap * D * 4; }
    __host__ __device__ static uint32_t off_p(uint32_t cap) { return off_q(cap) + kShortQ * D * 4; }
    __host__ __device__ static uint32_t bytes(uint32_t cap) { return off_p(cap) + kShortQ * cap * 4; }
};

template <int D>
__global__ void __launch_bounds__(kShortThreads) attention_short_kernel(AttnP p, uint32_t cap, int* error) {
    pdl_enter();
    using P = ShortPlan<D>;
    extern __shared__ __align__(16) unsigned char smem[];
    float* ks = reinterpret_cast<float*>(smem);
    float* vs = reinterpret_cast<float*>(smem + P::off_v(cap));
    float* qs = reinterpret_cast<float*>(smem + P::off_q(cap));
    float* ps = reinterpret_cast<float*>(smem + P::off_p(cap));
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

    // 1. scores (masked keys -inf), one key per thread
    uint64_t qlo[kShortQ], qhi[kShortQ];
#pragma unroll
    for (int qi = 0; qi < kShortQ; qi++) {
        key_range(p, p.qpos0 + q0 + qi, qlo[qi], qhi[qi]);
        if (qi >= nq) qlo[qi] = qhi[qi] = 0;
    }
    for (int j = threadIdx.x; j < n; j += kShortThreads) {
        float acc[kShortQ];
#pragma unroll
        for (int qi = 0; qi < kShortQ; qi++) acc[qi] = 0.0f;
        const float4* kr = reinterpret_cast<const float4*>(ks + j * P::kKStride);
#pragma unroll 4
        for (int c = 0; c < C4; c++) {
            const float4 kk = kr[c];
#pragma unroll
            for (int qi = 0; qi < kShortQ; qi++) {
                const float4 qq = reinterpret_cast<const float4*>(qs + qi * D)[c];
                acc[qi] += qq.x * kk.x + qq.y * kk.y + qq.z * kk.z + qq.w * kk.w;
            }
        }
        const uint64_t key = span_lo + j;
#pragma unroll
        for (int qi = 0; qi < kShortQ; qi++)
            ps[qi * cap + j] = (key >= qlo[qi] && key < qhi[qi]) ? acc[qi] * p.scale : ninf;
    }
    __syncthreads();

    // 2. softmax of row `warp`: weights e / sum, all zero for a row with no admitted key
    {
        const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
        float* row = ps + warp * cap;
        float m = ninf;
        for (int j = lane; j < n; j += 32) m = fmaxf(m, row[j]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (m == ninf) {
            for (int j = lane; j < n; j += 32) row[j] = 0.0f;
        } else {
            float l = 0.0f;
            for (int j = lane; j < n; j += 32) {
                const float e = expf(row[j] - m);
                row[j] = e;
                l += e;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
            for (int j = lane; j < n; j += 32) row[j] = row[j] / l;
        }
    }
    __syncthreads();

    // 3. out = P.V, one output column per thread, QPT queries each
    constexpr int QPT = kShortQ * D / kShortThreads;
    static_assert(QPT >= 1 && kShortThreads % D == 0, "one column per thread");
    const int d = threadIdx.x % D, qg = threadIdx.x / D;
    float acc0[QPT], acc1[QPT];
#pragma unroll
    for (int i = 0; i < QPT; i++) acc0[i] = acc1[i] = 0.0f;
    int j = 0;
    for (; j + 1 < n; j += 2) {
        const float v0 = vs[j * D + d], v1 = vs[(j + 1) * D + d];
#pragma unroll
        for (int i = 0; i < QPT; i++) {
            const float* prow = ps + (qg * QPT + i) * cap;
            acc0[i] += prow[j] * v0;
            acc1[i] += prow[j + 1] * v1;
        }
    }
    if (j < n) {
        const float v0 = vs[j * D + d];
#pragma unroll
        for (int i = 0; i < QPT; i++) acc0[i] += ps[(qg * QPT + i) * cap + j] * v0;
    }
#pragma unroll
    for (int i = 0; i < QPT; i++) {
        const int qi = qg * QPT + i;
        if (qi < nq) p.out[((q0 + qi) * p.head_count + head) * D + d] = acc0[i] + acc1[i];
    }
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
