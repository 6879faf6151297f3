// The int8 / elementwise side kernels the reference ships next to the INT4 path.
//
//   gemv_int8   out[r] = sum_k (q[r][k] * s[r][k/64] + b[r][k/64]) * x[k] with 8-bit affine G64
//               weights (shaders/GemvInt8.hlsl:13-33, row dot shaders/Common.hlsli:225-269; the
//               reference uses it for 8-bit router projections). HBM-bound at 1.03 B/weight:
//               one warp per row, each lane streaming 16 weights per 16-byte load with four
//               loads in flight, scale and bias per 64-group in fp32, a warp sum per row.
//   attn_gate   out = ctx * sigmoid(gate) elementwise over `batch` rows with strides
//               (shaders/AttnGate.hlsl:15-32, src/cpu_reference.cpp:550-556);
//               sigmoid(g) = 1 / (1 + exp(-g)) as shaders/Common.hlsli:157-159 computes it.
#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"

#include <algorithm>

namespace g4b {
namespace {

__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__global__ void __launch_bounds__(256) gemv_int8_kernel(const uint8_t* __restrict__ W, const uint16_t* __restrict__ S,
                                                        const uint16_t* __restrict__ B, const float* __restrict__ x,
                                                        float* __restrict__ out, int rows, int K) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= rows) return;  // warp-uniform
    const int gpr = K / 64;
    const uint4* wr = reinterpret_cast<const uint4*>(W + (size_t)row * K);
    const uint16_t* sr = S + (size_t)row * gpr;
    const uint16_t* br = B + (size_t)row * gpr;
    float acc = 0.f;
    // Lane l covers weights [16l, 16l + 16) of every 512-wide stretch; 4 stretches per trip.
    for (int base = 0; base < K; base += 4 * 512) {
        uint4 q[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int c = base + u * 512 + lane * 16;
            if (c < K) q[u] = ld_stream(wr + c / 16);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int c = base + u * 512 + lane * 16;
            if (c >= K) continue;
            const float s = bf16_to_f32(sr[c / 64]), b = bf16_to_f32(br[c / 64]);
            const float4* xv = reinterpret_cast<const float4*>(x + c);
            const uint32_t words[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
#pragma unroll
            for (int wdx = 0; wdx < 4; ++wdx) {
                const float4 xx = xv[wdx];
                const uint32_t p = words[wdx];
                acc += ((float)(p & 0xFFu) * s + b) * xx.x;
                acc += ((float)((p >> 8) & 0xFFu) * s + b) * xx.y;
                acc += ((float)((p >> 16) & 0xFFu) * s + b) * xx.z;
                acc += ((float)(p >> 24) * s + b) * xx.w;
            }
        }
    }
    acc = warp_sum(acc);
    if (lane == 0) out[row] = acc;
}

__global__ void attn_gate_kernel(const float* __restrict__ ctx, const float* __restrict__ gate, float* __restrict__ out,
                                 int n, int batch, int ctx_stride, int gate_stride, int out_stride) {
    const long long total = (long long)n * batch;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int m = (int)(i / n), c = (int)(i % n);
        const float g = gate[(size_t)m * gate_stride + c];
        const float sig = 1.0f / (1.0f + expf(-g));
        out[(size_t)m * out_stride + c] = ctx[(size_t)m * ctx_stride + c] * sig;
    }
}

}  // namespace

cudaError_t gemv_int8_launch(const uint8_t* W, const uint16_t* S, const uint16_t* B, const float* x, float* out,
                             int rows, int K, cudaStream_t st) {
    gemv_int8_kernel<<<(rows + 7) / 8, 256, 0, st>>>(W, S, B, x, out, rows, K);
    return cudaGetLastError();
}

cudaError_t attn_gate_launch(const float* ctx, const float* gate, float* out, int n, int batch, int ctx_stride,
                             int gate_stride, int out_stride, cudaStream_t st) {
    const long long total = (long long)n * batch;
    const int blocks = (int)std::min<long long>(148 * 8, (total + 255) / 256);
    attn_gate_kernel<<<blocks, 256, 0, st>>>(ctx, gate, out, n, batch, ctx_stride, gate_stride, out_stride);
    return cudaGetLastError();
}

}  // namespace g4b
