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

__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Activation rows a quad thread t holds in the digit modes (format 5 of common.cuh).
template <int NT>
struct DigitRows {
    static constexpr int J = (NT == 6 || NT == 4) ? 4 : 2;
};

// Digit modes (M = 5..16): one k-tile for one warp, 4 row tiles x 128 k. The nibble words of
// step kk give the m16n8k32 A operand directly: even nibbles (k = 8t + 0, 2, 4, 6) and odd
// nibbles (k = 8t + 1, 3, 5, 7) of rows g and g+8, each as four u8 lanes. Per 64-group the
// int32 digit sums are folded into P = sum q v in fp32 and acc += E * (s * P + b * Y).
// acc[r][j][h]: row tile r, the thread's j-th activation row, weight row g + 8h.
template <int NT>
__device__ __forceinline__ void compute_ktile_digits(const uint4* __restrict__ blk, const uint2* __restrict__ bsm,
                                                     const float2* __restrict__ gsm,
                                                     float (&acc)[kTilesPerWarp][DigitRows<NT>::J][2], int lane) {
    constexpr uint32_t kLo = 0x0F0F0F0Fu;
    constexpr int J = DigitRows<NT>::J;
    const int t = lane & 3;
    uint4 nib[kTilesPerWarp][2], sb[kTilesPerWarp];
#pragma unroll
    for (int r = 0; r < kTilesPerWarp; ++r) {
        nib[r][0] = blk[(r * 2 + 0) * 32 + lane];
        nib[r][1] = blk[(r * 2 + 1) * 32 + lane];
        sb[r] = blk[256 + r * 8 + (lane >> 2)];
    }
#pragma unroll
    for (int G = 0; G < 2; ++G) {
        int ci[kTilesPerWarp][NT][4];
#pragma unroll
        for (int r = 0; r < kTilesPerWarp; ++r)
#pragma unroll
            for (int n = 0; n < NT; ++n) ci[r][n][0] = ci[r][n][1] = ci[r][n][2] = ci[r][n][3] = 0;
#pragma unroll
        for (int kq = 0; kq < 2; ++kq) {
            const int kk = 2 * G + kq;
            uint2 bf[NT];
#pragma unroll
            for (int n = 0; n < NT; ++n) bf[n] = bsm[(kk * NT + n) * 32 + lane];
#pragma unroll
            for (int r = 0; r < kTilesPerWarp; ++r) {
                const uint4& h = nib[r][G];
                const uint32_t w0 = kq ? h.z : h.x, w8 = kq ? h.w : h.y;
                const uint32_t a0 = w0 & kLo, a1 = w8 & kLo, a2 = (w0 >> 4) & kLo, a3 = (w8 >> 4) & kLo;
#pragma unroll
                for (int n = 0; n < NT; ++n) mma_u8s8(ci[r][n], a0, a1, a2, a3, bf[n].x, bf[n].y);
            }
        }
        // Group epilogue. Digit columns of the thread's rows (digit_col in common.cuh):
        // row t: (tile 3b, cols 2t, 2t+1) = d0, d1; (tile 3b+1, col 2t) = d2
        // row 4+t: (tile 3b+1, col 2t+1) = d0; (tile 3b+2, cols 2t, 2t+1) = d1, d2
        // two tiles: row 4 in (tile 1, col 2d+1) of thread d, gathered by shuffles;
        // four tiles: rows 8, 9 in (tile 3, cols 2d, 2d+1) of thread d, gathered the same way.
        float2 ey[J];
#pragma unroll
        for (int j = 0; j < J; ++j) {
            const int m = (NT == 2 && j == 1) ? 4 : (NT == 4 && j >= 2) ? 6 + j : 4 * j + t;
            ey[j] = gsm[G * kMaxM + m];
        }
#pragma unroll
        for (int r = 0; r < kTilesPerWarp; ++r) {
            const uint32_t sbg = G ? sb[r].z : sb[r].x, sbg8 = G ? sb[r].w : sb[r].y;
            const float sc[2] = {bf16_lo(sbg), bf16_lo(sbg8)}, bi[2] = {bf16_hi(sbg), bf16_hi(sbg8)};
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float P[J];
#pragma unroll
                for (int b = 0; b < (NT == 6 ? 2 : 1); ++b) {
                    P[2 * b] = fmaf((float)ci[r][3 * b + 1][2 * h], 65536.0f,
                                    (float)(ci[r][3 * b][2 * h] + 256 * ci[r][3 * b][2 * h + 1]));
                    if (NT >= 3)
                        P[2 * b + 1] = fmaf((float)ci[r][3 * b + 2][2 * h + 1], 65536.0f,
                                            (float)(ci[r][3 * b + 1][2 * h + 1] + 256 * ci[r][3 * b + 2][2 * h]));
                }
                if constexpr (NT == 2) {
                    const int c = ci[r][1][2 * h + 1];  // thread d holds digit d of row 4
                    const int c1 = __shfl_down_sync(0xffffffffu, c, 1), c2 = __shfl_down_sync(0xffffffffu, c, 2);
                    P[1] = fmaf((float)c2, 65536.0f, (float)(c + 256 * c1));
                }
                if constexpr (NT == 4) {
#pragma unroll
                    for (int q = 0; q < 2; ++q) {  // thread d holds digit d of rows 8 (q = 0) and 9
                        const int c = ci[r][3][2 * h + q];
                        const int c1 = __shfl_down_sync(0xffffffffu, c, 1), c2 = __shfl_down_sync(0xffffffffu, c, 2);
                        P[2 + q] = fmaf((float)c2, 65536.0f, (float)(c + 256 * c1));
                    }
                }
#pragma unroll
                for (int j = 0; j < J; ++j)
                    acc[r][j][h] = fmaf(ey[j].x, fmaf(bi[h], ey[j].y, sc[h] * P[j]), acc[r][j][h]);
            }
        }
    }
}

}  // namespace g4b
