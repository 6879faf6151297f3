// Host interface of the verify GEMM (vgemm.cu).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

struct VgemmParams {
    const void* w;        // vgemm-layout weights, n_wrg * ktiles blocks of 4608 B
    const uint4* bfrag;   // B fragments of the activations, [K/32][nb][32]
    const float2* gsum;   // {E, Y} per (64-group, column), [K/64][nacc][8]
    float* out;           // [M][ldo] fp32
    int ldo;
    int N;                // output rows (unpadded)
    int M;                // activation rows, 1..16
    int n_wrg;            // ceil(N / 64)
    int n_crg;            // ceil(n_wrg / 4): 256-row CTA row groups
    int ktiles;           // ceil(K / 128)
    float* part;          // split-K scratch: [n_crg][max_slots][16][256] fp32
    int* counters;        // [n_crg] arrival counters, zero between launches
    int max_slots;
};

// Grid size (CTAs) for a launch: all resident at once, never more than the unit count.
int vgemm_grid(int M, int n_crg, int ktiles);
// Split-K slots per row group needed for `grid` CTAs.
int vgemm_max_slots(int grid, int n_crg, int ktiles);
cudaError_t vgemm_launch(const VgemmParams& p, int grid, cudaStream_t st, bool pdl);
