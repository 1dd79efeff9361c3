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

}  // namespace

namespace k {

bool attention_tc_eligible(const AttentionArgs& a);
mg_status attention_tc(Device* d, const AttentionArgs& a);

mg_status attention(Device* d, const AttentionArgs& a) {
    if (a.seq_len == 0 || a.head_count == 0) return MG_OK;
    if (attention_tc_eligible(a)) return attention_tc(d, a);
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
    if (a.seq_len == 0 || a.head_count == 0) return MG_OK;
    const bool aligned = ((reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.k) |
                           reinterpret_cast<uintptr_t>(a.v) | reinterpret_cast<uintptr_t>(a.out)) & 15) == 0 &&
                         a.q_model_dim % 4 == 0 && a.kv_model_dim % 4 == 0 && a.v_model_dim % 4 == 0;
    const bool tiled = aligned && a.value_dim == a.head_dim && (a.head_dim == 64 || a.head_dim == 128 ||
                                                                 a.head_dim == 32 || a.head_dim == 16);
    if (tiled) {
        dim3 grid((unsigned)((a.seq_len + BQ - 1) / BQ), (unsigned)a.head_count);
        if (a.head_count > 65535) return fail(MG_SHAPE_UNSUPPORTED, "attention head_count exceeds the launch grid");
        switch (a.head_dim) {
            case 16: attention_tile_kernel<1><<<grid, kAttnThreads, 0, d->stream>>>(p); break;
            case 32: attention_tile_kernel<2><<<grid, kAttnThreads, 0, d->stream>>>(p); break;
            case 64: attention_tile_kernel<4><<<grid, kAttnThreads, 0, d->stream>>>(p); break;
            default: attention_tile_kernel<8><<<grid, kAttnThreads, 0, d->stream>>>(p); break;
        }
        return launched(d, "attention kernel launch");
    }
    const uint64_t warps = a.head_count * a.seq_len;
    const uint64_t blocks = (warps + 7) / 8;
    if (blocks > 0x7FFFFFFFull) return fail(MG_SHAPE_UNSUPPORTED, "attention launch size overflows");
    attention_generic_kernel<<<(unsigned)blocks, 256, 0, d->stream>>>(p);
    return launched(d, "attention kernel launch");
}

}  // namespace k
}  // namespace mg
