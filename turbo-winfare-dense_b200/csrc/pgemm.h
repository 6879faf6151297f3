// Host interface of the prefill GEMM (pgemm.cu): out[m][n] = sum_k (q[n][k] * s[n][k/64] +
// b[n][k/64]) * x[m][k] for 17..128 activation rows on the tcgen05 tensor cores.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

struct PgemmParams {
    const void* w;      // prefill-layout weights: [n_tiles][K/64][4608 B]
    const void* act;    // wide-layout activations (common.cuh, format 4)
    int g_layout;       // 64-groups the activation buffer was laid out for (K rounded up to 128)
    float* y;           // dense output y[m * ldy + n]
    int ldy;
    float* part;        // split-K slots [n_tiles][max_slots][128 cols][128 rows]
    unsigned* cnt;      // [n_tiles] arrival counters, zero before a launch and after it
    int N, K, M;        // rows, inner dimension (multiple of 64), activation rows (1..128)
    int n_tiles;        // ceil(N / 128)
    int max_slots;      // pgemm_max_slots(n_tiles, K / 64, grid)
    int* err;           // set non-zero if a bounded wait gave up
};

constexpr int kPgemmTileRows = 128;
constexpr int kPgemmBlockBytes = 4608;  // one (128-row tile, 64-group) block

inline int pgemm_n_tiles(int N) { return (N + kPgemmTileRows - 1) / kPgemmTileRows; }
inline size_t pgemm_weight_bytes(int N, int K) { return (size_t)pgemm_n_tiles(N) * (K / 64) * kPgemmBlockBytes; }
// CTAs of a launch on this device: one per SM, never more than the unit count.
int pgemm_grid(int n_tiles, int groups);
// Split-K slots a tile can need with `grid` CTAs.
int pgemm_max_slots(int n_tiles, int groups, int grid);
inline size_t pgemm_part_floats(int n_tiles, int max_slots) {
    return (size_t)n_tiles * max_slots * kPgemmTileRows * 128;
}

// Container row-major W [N][K/8] u32, S/B [N][K/64] bf16 -> prefill layout.
cudaError_t pgemm_repack(const uint32_t* W, const uint16_t* S, const uint16_t* B, int N, int K, void* out,
                         cudaStream_t st);
cudaError_t pgemm_launch(const PgemmParams& p, cudaStream_t st, bool pdl);
