// Portable f32 matmul on the CUDA cores: any shape, either operand transposed, any
// alignment.  It serves the shapes the tensor-core and GEMV paths do not take (odd row
// strides, transposed operands at few rows) and is the in-library cross-check of those
// paths.  Every output accumulates k in ascending order as the reference's
// `matmul_kernel` does (src/kernels.cu:1265-1294); 64x64 tiles, 4x4 outputs per thread.
#include "internal.h"

namespace mg {
namespace {

constexpr int BM = 64, BN = 64, BK = 16;

__global__ void __launch_bounds__(256) gemm_simt_kernel(k::GemmArgs g) {
    pdl_enter();
    __shared__ float As[BK][BM + 4];
    __shared__ float Bs[2][BK][BN + 4];
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    const uint64_t row0 = (uint64_t)blockIdx.y * BM, col0 = (uint64_t)blockIdx.x * BN;
    const int nb = g.gated ? 2 : 1;
    float acc[2][4][4] = {};
    for (uint64_t k0 = 0; k0 < g.k; k0 += BK) {
        for (int i = threadIdx.x; i < BM * BK; i += 256) {
            int r = i / BK, kk = i % BK;
            uint64_t gr = row0 + r, gk = k0 + kk;
            float v = 0.0f;
            if (gr < g.m && gk < g.k) v = g.transpose_a ? g.a[gk * g.m + gr] : g.a[gr * g.k + gk];
            As[kk][r] = v;
        }
        for (int z = 0; z < nb; z++) {
            const float* w = z ? g.b2 : g.b;
            for (int i = threadIdx.x; i < BN * BK; i += 256) {
                int kk = i / BN, c = i % BN;
                uint64_t gk = k0 + kk, gc = col0 + c;
                float v = 0.0f;
                if (gk < g.k && gc < g.n) v = g.transpose_b ? w[gc * g.k + gk] : w[gk * g.n + gc];
                Bs[z][kk][c] = v;
            }
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < BK; kk++) {
            float av[4], bv[4];
#pragma unroll
            for (int i = 0; i < 4; i++) av[i] = As[kk][ty * 4 + i];
            for (int z = 0; z < nb; z++) {
#pragma unroll
                for (int j = 0; j < 4; j++) bv[j] = Bs[z][kk][tx * 4 + j];
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int j = 0; j < 4; j++) acc[z][i][j] += av[i] * bv[j];
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint64_t r = row0 + ty * 4 + i;
        if (r >= g.m) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const uint64_t c = col0 + tx * 4 + j;
            if (c >= g.n) continue;
            float s = acc[0][i][j];
            if (g.gated) {
                s = (s * (1.0f / (1.0f + expf(-s)))) * acc[1][i][j];
            } else if (g.addend_mode == 1) {
                s += g.addend[c];
            } else if (g.addend_mode == 2) {
                s += g.addend[r * g.n + c];
            }
            g.out[r * g.n + c] = s;
        }
    }
}

}  // namespace

namespace k {

mg_status gemm_simt(Device* d, const GemmArgs& g) {
    dim3 grid((unsigned)((g.n + BN - 1) / BN), (unsigned)((g.m + BM - 1) / BM));
    if (grid.y > 65535) return fail(MG_SHAPE_UNSUPPORTED, "matmul with %llu rows exceeds the launch grid", (unsigned long long)g.m);
    enqueue(d, gemm_simt_kernel, grid, 256, 0, g);
    return launched(d, "matmul kernel launch");
}

}  // namespace k
}  // namespace mg
