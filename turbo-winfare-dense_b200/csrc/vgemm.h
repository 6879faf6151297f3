// Host and device interface of the verify GEMM (vgemm.cu).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

// Split-K partial output of one GEMM launch: part[n_crg][max_slots][16][256] fp32. Output
// element (m, n) is the sum, in slot order, of part[n/256][s][m][n%256] over the slots of
// the CTAs whose unit ranges meet row group n/256.
struct PartView {
    float* part;
    int max_slots;
    int n_crg;
    int ktiles;
    int grid;
};

struct VgemmParams {
    const void* w;        // vgemm-layout weights: [n_crg][ktiles][4 warps][4608 B]
    const uint4* bfrag;   // B fragments of the activations, [K/32][nb][32]
    const float2* gsum;   // {E, Y} per (64-group, column), [K/64][nacc][8]
    PartView out;         // split-K partial slots (scratch when y is set)
    int N;                // output rows (unpadded)
    int M;                // activation rows, 1..16
    int n_wrg;            // ceil(N / 64)
    int* err;             // set non-zero if a bounded wait gave up
    // Dense output y[m * ldy + n] (optional). When set, the kernel finishes the split-K sum
    // itself: a row group covered by one CTA is written directly; otherwise the last CTA to
    // arrive on the group's counter (cnt[crg], zero before the launch and left zero after it)
    // adds the slots in slot order. When null, only the partial slots are written.
    float* y;
    int ldy;
    unsigned* cnt;        // [n_crg] arrival counters
};

// CTA row group (256 rows) count and k-tile count for an [N][K] matrix.
inline int vgemm_n_crg(int N) { return (N + 255) / 256; }
inline int vgemm_ktiles(int K) { return (K + 127) / 128; }
// Bytes of the repacked weights (padded to whole CTA row groups).
inline size_t vgemm_weight_bytes(int N, int K) {
    return (size_t)vgemm_n_crg(N) * vgemm_ktiles(K) * 4 * 4608;
}
// Grid size (CTAs) for a launch: all resident at once, never more than the unit count.
int vgemm_grid(int M, int n_crg, int ktiles);
// Split-K slots per row group needed for `grid` CTAs.
int vgemm_max_slots(int grid, int n_crg, int ktiles);
// Slots a launch with this grid needs at most over every M it will be run with.
int vgemm_plan_slots(int n_crg, int ktiles);
cudaError_t vgemm_launch(const VgemmParams& p, cudaStream_t st, bool pdl);

#ifdef __CUDACC__
// The CTA whose unit range [c*T/G, (c+1)*T/G) holds unit x. 32-bit arithmetic:
// vgemm_launch rejects launches where (T+1)*G could reach 2^31.
__device__ __forceinline__ int vgemm_cta_of_unit32(int x, int T, int G) { return ((x + 1) * G + T - 1) / T - 1; }
#endif
