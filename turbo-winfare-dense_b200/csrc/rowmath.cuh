// Scalar numerics of the row kernels (rowops.cu), each restating the reference's CPU arithmetic.
#pragma once
#include <cstdint>

namespace g4b {

// FP16 round trip of the reference oracle (src/cpu_reference.cpp:51-84): round to nearest
// even for normal halves, values below the smallest normal half become signed zero, values
// at or above 2^16 become infinity. Returns the half's bit pattern.
__device__ __forceinline__ uint16_t f16_bits_like_reference(float f) {
    const uint32_t x = __float_as_uint(f);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const int e = (int)((x >> 23) & 0xFFu) - 127 + 15;
    const uint32_t man = x & 0x7FFFFFu;
    if (e <= 0) return (uint16_t)sign;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    const uint32_t round_bit = (man >> 12) & 1u;
    const uint32_t sticky = (man & 0xFFFu) != 0u;
    uint32_t v = sign | ((uint32_t)e << 10) | (man >> 13);
    if (round_bit && (sticky || (v & 1u))) ++v;
    return (uint16_t)v;
}

__device__ __forceinline__ uint16_t bf16_bits_rne(float f) {
    uint32_t u = __float_as_uint(f);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

// 1 / sqrt(mean + eps) with IEEE sqrt and division, as the reference computes it.
__device__ __forceinline__ float inv_rms(float sumsq, int n) {
    return 1.0f / sqrtf(sumsq / (float)n + 1e-6f);
}

// gelu_tanh(x) = 0.5 x (1 + tanh(0.7978845608 (x + 0.044715 x^3))) (shaders/Common.hlsli:145-149,
// src/cpu_reference.cpp:568-581)
__device__ __forceinline__ float gelu_tanh_dev(float x) {
    const float k = 0.7978845608028654f;
    const float inner = k * (x + 0.044715f * x * x * x);
    return 0.5f * x * (1.0f + tanhf(inner));
}

}  // namespace g4b
