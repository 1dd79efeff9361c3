// The rotary-embedding rotation of one (position, pair), shared by the rope kernels and the
// tensor-core GEMM's fused RoPE epilogue: the reference's per-pair expression
// (src/kernels.cu:1183-1228) -- powf of the base, optional banded (Llama 3) or YaRN frequency
// scaling, cosf / sinf of position x frequency, partial rotation.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mg {

struct RopeK {
    uint64_t rows, cols, half, dimension, position_offset, head_count, head_width, rotated_pairs;
    float base, scale, banded_factor, low_freq_factor, high_freq_factor, original_context_length;
    float yarn_factor, yarn_low, yarn_high, amplitude;
    int half_split;
    int vec;  // 1: 16-byte path (alignment and divisibility checked on the host)
    const uint64_t* step;  // a captured step's advancing position offset (null: none)
};

__device__ __forceinline__ float2 rope_cs(const RopeK& p, uint64_t row, uint64_t pair) {
    const uint64_t offset = p.position_offset + (p.step ? *p.step : 0);
    float position = (float)(offset + row) * p.scale;
    float frequency = powf(p.base, -2.0f * (float)pair / (float)p.dimension);
    if (p.banded_factor > 0.0f) {
        float wavelength = 6.283185307179586f / frequency;
        if (wavelength < p.original_context_length / p.high_freq_factor) {
        } else if (wavelength > p.original_context_length / p.low_freq_factor) {
            frequency = frequency / p.banded_factor;
        } else {
            float smooth = (p.original_context_length / wavelength - p.low_freq_factor) /
                           (p.high_freq_factor - p.low_freq_factor);
            frequency = (1.0f - smooth) * frequency / p.banded_factor + smooth * frequency;
        }
    }
    if (p.yarn_factor > 0.0f) {
        float high = p.yarn_low == p.yarn_high ? p.yarn_high + 0.001f : p.yarn_high;
        float ramp = ((float)pair - p.yarn_low) / (high - p.yarn_low);
        ramp = fminf(fmaxf(ramp, 0.0f), 1.0f);
        float interpolated = frequency / p.yarn_factor;
        frequency = interpolated * ramp + frequency * (1.0f - ramp);
    }
    float angle = pair < p.rotated_pairs ? position * frequency : 0.0f;
    float amp = pair < p.rotated_pairs ? p.amplitude : 1.0f;
    return make_float2(cosf(angle) * amp, sinf(angle) * amp);
}

}  // namespace mg
