// The verify GEMM's per-warp k-tile step (vgemm.cu): one warp multiplies its 64 rows x 128 k of
// INT4 weights (one 4608-byte block of the vgemm layout, in shared memory) by the activation
// fragments of that k-tile and adds the result into fp32 accumulators.
#pragma once
#include "common.cuh"

namespace g4b {

__device__ __forceinline__ void mma16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1, const float* c) {
    // Not volatile: the MMA has no side effects, and letting the compiler interleave
    // independent row tiles hides the tensor pipe's fixed latency.
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]),
          "f"(c[3]));
}

// k-tiles of activation fragments per staged chunk: 8 KB of fragments per chunk.
template <int NB>
struct Chunk {
    static constexpr int kt = 4 / NB > 0 ? 4 / NB : 1;
    static constexpr int frag_u4 = kt * 4 * NB * 32;
};

// One k-tile for one warp: 4 row tiles x 128 k, weights from the shared-memory ring.
template <int NB, int NACC, bool PACKED>
__device__ __forceinline__ void compute_ktile(const uint4* __restrict__ blk, const uint4* __restrict__ bsm,
                                              const float4* __restrict__ gsm,
                                              float (&acc)[kTilesPerWarp][NACC][4], int lane) {
    constexpr uint32_t M0 = 0x000F000Fu, M1 = 0x00F000F0u;
    const float zero[4] = {0.f, 0.f, 0.f, 0.f};
    uint4 nib[kTilesPerWarp][2], sb[kTilesPerWarp];
#pragma unroll
    for (int r = 0; r < kTilesPerWarp; ++r) {
        nib[r][0] = blk[(r * 2 + 0) * 32 + lane];
        nib[r][1] = blk[(r * 2 + 1) * 32 + lane];
        sb[r] = blk[256 + r * 8 + (lane >> 2)];
    }
    float P[kTilesPerWarp][NACC][4];
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
        uint4 bf[NB];
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) bf[nb] = bsm[(kk * NB + nb) * 32 + lane];
        const bool first = (kk & 1) == 0;
        // Row tiles innermost: consecutive MMAs are independent, so the four accumulation
        // chains of a warp overlap in the tensor pipe.
#pragma unroll
        for (int step = 0; step < 2; ++step) {
#pragma unroll
            for (int part = 0; part < (PACKED ? 1 : 2); ++part) {
#pragma unroll
                for (int a = 0; a < NACC; ++a) {
                    const uint4& b = bf[PACKED ? 0 : 2 * a + part];
                    const uint32_t b0 = step ? b.z : b.x, b1 = step ? b.w : b.y;
#pragma unroll
                    for (int r = 0; r < kTilesPerWarp; ++r) {
                        const uint4& h = nib[r][kk >> 1];
                        uint32_t wg = (kk & 1) ? h.z : h.x;
                        uint32_t wg8 = (kk & 1) ? h.w : h.y;
                        if (step) { wg >>= 8; wg8 >>= 8; }
                        // step 0: k slots {0,4} and 16x{1,5}; step 1: {2,6} and 16x{3,7}
                        mma16816(P[r][a], wg & M0, wg8 & M0, wg & M1, wg8 & M1, b0, b1,
                                 (first && step == 0 && part == 0) ? zero : P[r][a]);
                    }
                }
            }
        }
        if (kk & 1) {
            // group epilogue: acc += E * (s * P + b * Y), per row (s, b) and per column (E, Y)
            const int G = kk >> 1;
#pragma unroll
            for (int a = 0; a < NACC; ++a) {
                const float4 ey = gsm[(G * NACC + a) * 4 + (lane & 3)];  // {E0, Y0, E1, Y1}
#pragma unroll
                for (int r = 0; r < kTilesPerWarp; ++r) {
                    const uint32_t sbg = G ? sb[r].z : sb[r].x;
                    const uint32_t sbg8 = G ? sb[r].w : sb[r].y;
                    const float s0 = bf16_lo(sbg), b0 = bf16_hi(sbg);
                    const float s8 = bf16_lo(sbg8), b8 = bf16_hi(sbg8);
                    acc[r][a][0] = fmaf(ey.x, fmaf(b0, ey.y, s0 * P[r][a][0]), acc[r][a][0]);
                    acc[r][a][1] = fmaf(ey.z, fmaf(b0, ey.w, s0 * P[r][a][1]), acc[r][a][1]);
                    acc[r][a][2] = fmaf(ey.x, fmaf(b8, ey.y, s8 * P[r][a][2]), acc[r][a][2]);
                    acc[r][a][3] = fmaf(ey.z, fmaf(b8, ey.w, s8 * P[r][a][3]), acc[r][a][3]);
                }
            }
        }
    }
}

}  // namespace g4b
