// Load-time repack of a container INT4 G64 matrix into the vgemm layout (common.cuh).
// Source is the container's row-major form: W [N][K/8] u32, S/B [N][K/64] bf16
// (src/cpu_reference.cpp:367-381). Runs once per matrix on the device.
#include "common.cuh"
#include "kernels.h"

namespace g4b {

// Block index of warp row group wrg (= 4*crg + w) at k-tile kt: [crg][kt][w].
__device__ __forceinline__ long long block_index(long long wrg, int kt, int ktiles) {
    return ((wrg >> 2) * ktiles + kt) * 4 + (wrg & 3);
}

// One thread per (row group, k-tile, r, half, lane) output uint4; n_wrg is padded to whole
// 256-row CTA groups and rows past N are zero.
__global__ void repack_nibbles(const uint32_t* __restrict__ W, int N, int K, int ktiles, int n_wrg,
                               uint4* __restrict__ out) {
    const long long total = (long long)n_wrg * ktiles * 256;
    const int wpr = K / 8;  // words per source row
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int lane = (int)(i & 31);
        const int half = (int)((i >> 5) & 1);
        const int r = (int)((i >> 6) & 3);
        const long long blk = i >> 8;  // wrg * ktiles + kt
        const int kt = (int)(blk % ktiles);
        const long long wrg = blk / ktiles;
        const int g = lane >> 2, t = lane & 3;
        const long long row0 = wrg * 64 + r * 16 + g, row8 = row0 + 8;
        uint32_t v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int kk = 2 * half + (j >> 1);
            const long long row = (j & 1) ? row8 : row0;
            const int word = kt * 16 + kk * 4 + t;
            v[j] = (row < N && word < wpr) ? W[row * wpr + word] : 0u;
        }
        out[block_index(wrg, kt, ktiles) * (kKTileBytes / 16) + (r * 2 + half) * 32 + lane] =
            make_uint4(v[0], v[1], v[2], v[3]);
    }
}

// One thread per (row group, k-tile, r, g) scale/bias uint4.
__global__ void repack_scales(const uint16_t* __restrict__ S, const uint16_t* __restrict__ B, int N, int K,
                              int ktiles, int n_wrg, uint4* __restrict__ out) {
    const long long total = (long long)n_wrg * ktiles * 32;
    const int gpr = K / 64;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int g = (int)(i & 7);
        const int r = (int)((i >> 3) & 3);
        const long long blk = i >> 5;
        const int kt = (int)(blk % ktiles);
        const long long wrg = blk / ktiles;
        const long long row0 = wrg * 64 + r * 16 + g, row8 = row0 + 8;
        uint32_t v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int grp = kt * 2 + (j >> 1);
            const long long row = (j & 1) ? row8 : row0;
            uint32_t s = 0, b = 0;
            if (row < N && grp < gpr) {
                s = S[row * gpr + grp];
                b = B[row * gpr + grp];
            }
            v[j] = s | (b << 16);
        }
        out[block_index(wrg, kt, ktiles) * (kKTileBytes / 16) + 256 + r * 8 + g] = make_uint4(v[0], v[1], v[2], v[3]);
    }
}

}  // namespace g4b

size_t g4b_qmat_bytes(int N, int K) {
    const int n_wrg = (N + 255) / 256 * 4, ktiles = (K + 127) / 128;
    return (size_t)n_wrg * ktiles * g4b::kKTileBytes;
}

cudaError_t g4b_repack(const uint32_t* W, const uint16_t* S, const uint16_t* B, int N, int K, void* out,
                       cudaStream_t st) {
    if (N <= 0 || K <= 0 || K % 64) return cudaErrorInvalidValue;
    const int n_wrg = (N + 255) / 256 * 4, ktiles = (K + 127) / 128;
    g4b::repack_nibbles<<<1184, 256, 0, st>>>(W, N, K, ktiles, n_wrg, reinterpret_cast<uint4*>(out));
    g4b::repack_scales<<<592, 256, 0, st>>>(S, B, N, K, ktiles, n_wrg, reinterpret_cast<uint4*>(out));
    return cudaGetLastError();
}
