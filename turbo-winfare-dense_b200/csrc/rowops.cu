// Row-wise kernels around the verify GEMM: fragment producers, RMSNorm + residual
// epilogues, GeGLU, embedding gather, Q/K/V epilogue with the FP16 KV-ring write.
#include "bfrag.cuh"
#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"

namespace g4b {

// Plain conversion: x [M][ldx] fp32 -> B fragments. One warp per (row, 64-group); groups
// past K (k-tile padding) are written as zeros.
__global__ void bfrag_from_f32_kernel(const float* __restrict__ x, int ldx, int M, int K, void* bfrag) {
    __shared__ __half stage[8][128];
    pdl_wait();
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int Kp = (K + 127) / 128 * 128;
    const int ngroups = Kp / 64;
    const BFragView v = bfrag_view(bfrag, Kp, M);
    const int total = M * ngroups;
    for (int w = blockIdx.x * 8 + wib; w < total; w += gridDim.x * 8) {
        const int m = w / ngroups, gi = w % ngroups;
        const int k = gi * 64 + 2 * lane;
        const float x0 = k < K ? x[(size_t)m * ldx + k] : 0.f;
        const float x1 = k + 1 < K ? x[(size_t)m * ldx + k + 1] : 0.f;
        bfrag_store_group(v, M, m, gi, x0, x1, stage[wib]);
    }
}

}  // namespace g4b

cudaError_t g4b_bfrag_from_f32(const float* x, int ldx, int M, int K, void* bfrag, cudaStream_t st, bool pdl) {
    const int ngroups = (K + 127) / 128 * 2;
    const int blocks = (M * ngroups + 7) / 8;
    return g4b::launch(g4b::bfrag_from_f32_kernel, dim3(blocks < 1184 ? blocks : 1184), dim3(256), 0, st, pdl, x,
                       ldx, M, K, bfrag);
}
