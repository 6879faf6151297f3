// Device-side synthetic weights with BASELINE config-0 value distributions, for model
// shapes too large to write as a container file per benchmark run (the 31B target is 17 GB).
// Values are a pure function of (seed, tensor id, GLOBAL element index), so every tensor-
// parallel rank generates exactly its own shard of the same logical model.
//   nibbles: uniform 0..15 (uniform random words), scales |N(0, 0.02)|, biases N(0, 0.01),
//   norm weights 1 + N(0, 0.05), all non-quantized values rounded to bf16.
#include <cstdint>
#include <cuda_runtime.h>

#include "synth.h"

namespace g4b {

__device__ __forceinline__ uint64_t mix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ULL;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ULL;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBULL;
    return x ^ (x >> 31);
}

__device__ __forceinline__ uint64_t key(uint64_t seed, uint64_t tensor, uint64_t idx) {
    return mix64(mix64(seed * 0x100000001B3ULL + tensor) ^ idx);
}

__device__ __forceinline__ float normal_from(uint64_t h) {
    const float u1 = ((float)((h >> 40) & 0xFFFFFF) + 1.0f) * (1.0f / 16777217.0f);
    const float u2 = (float)((h >> 16) & 0xFFFFFF) * (1.0f / 16777216.0f);
    return sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

__device__ __forceinline__ uint16_t bf16_rne(float f) {
    uint32_t u = __float_as_uint(f);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

// Local block rows [0, rows) x words [0, K/8) map to global rows row0+r and global word
// columns col0/8 + c of a logical [*, Kg] matrix.
__global__ void synth_qblock_kernel(uint32_t* W, uint16_t* S, uint16_t* B, int rows, int K, long long row0, int col0,
                                    int Kg, uint64_t seed, uint64_t tensor, int centered) {
    const long long nw = (long long)rows * (K / 8);
    const long long ng = (long long)rows * (K / 64);
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nw; i += stride) {
        const long long r = i / (K / 8), c = i % (K / 8);
        const long long gi = (row0 + r) * (Kg / 8) + col0 / 8 + c;
        W[i] = (uint32_t)(key(seed, tensor * 4 + 0, gi) >> 32);
    }
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < ng; i += stride) {
        const long long r = i / (K / 64), c = i % (K / 64);
        const long long gi = (row0 + r) * (Kg / 64) + col0 / 64 + c;
        const uint16_t s = bf16_rne(fabsf(normal_from(key(seed, tensor * 4 + 1, gi))) * 0.02f);
        float b = normal_from(key(seed, tensor * 4 + 2, gi)) * 0.01f;
        if (centered) b -= 7.5f * __uint_as_float((uint32_t)s << 16);
        S[i] = s;
        B[i] = bf16_rne(b);
    }
}

__global__ void synth_norm_kernel(uint16_t* out, int n, uint64_t seed, uint64_t tensor) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        out[i] = bf16_rne(1.0f + normal_from(key(seed, tensor, (uint64_t)i)) * 0.05f);
}

}  // namespace g4b

cudaError_t g4b_synth_qblock(uint32_t* W, uint16_t* S, uint16_t* B, int rows, int K, long long row0, int col0,
                             int Kg, uint64_t seed, uint64_t tensor, bool centered, cudaStream_t st) {
    g4b::synth_qblock_kernel<<<2048, 256, 0, st>>>(W, S, B, rows, K, row0, col0, Kg, seed, tensor, centered ? 1 : 0);
    return cudaGetLastError();
}

cudaError_t g4b_synth_norm(uint16_t* out, int n, uint64_t seed, uint64_t tensor, cudaStream_t st) {
    g4b::synth_norm_kernel<<<64, 256, 0, st>>>(out, n, seed, tensor);
    return cudaGetLastError();
}
