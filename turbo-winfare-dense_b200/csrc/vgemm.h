// Host and device interface of the verify GEMM (vgemm.cu).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

// Split-K partial output of one GEMM launch: part[n_crg][max_slots][16][256] fp32. Output
// element (m, n) is the sum, in slot order, of part[n/256][s][m][n%256] for
// s < nslots(n/256). Consumers reduce it with vgemm_part_get / vgemm_part_get4.
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
    PartView out;         // partial sums (always; consumers reduce the slots)
    int N;                // output rows (unpadded)
    int M;                // activation rows, 1..16
    int n_wrg;            // ceil(N / 64)
    int* err;             // set non-zero if a bounded wait gave up
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
// Reduces a PartView into out[m][n] (ldo floats per row).
cudaError_t vgemm_reduce(const PartView& v, int M, int N, float* out, int ldo, cudaStream_t st, bool pdl);

#ifdef __CUDACC__
__device__ __forceinline__ int vgemm_cta_of_unit(long long x, long long T, long long G) {
    return (int)(((x + 1) * G + T - 1) / T - 1);
}
// Same formula in 32-bit arithmetic: (x+1)*G stays below 2^31 for every launch this library
// makes (T = row groups x k-tiles < 2^17, G <= 16 x 148 CTAs).
__device__ __forceinline__ int vgemm_cta_of_unit32(int x, int T, int G) { return ((x + 1) * G + T - 1) / T - 1; }
__device__ __forceinline__ int vgemm_nslots(const PartView& v, int crg) {
    const int T = v.n_crg * v.ktiles;
    const int lo = vgemm_cta_of_unit32(crg * v.ktiles, T, v.grid);
    const int hi = vgemm_cta_of_unit32((crg + 1) * v.ktiles - 1, T, v.grid);
    return hi - lo + 1;
}
// Slot 0 of row m in CTA row group crg, and the slot count; slot s of column nl is at
// p[s * 4096 + nl].
struct SlotRow {
    const float* p;
    int ns;
};
__device__ __forceinline__ SlotRow vgemm_slot_row(const PartView& v, int m, int crg) {
    SlotRow r;
    r.p = v.part + ((size_t)crg * v.max_slots * 16 + m) * 256;
    r.ns = vgemm_nslots(v, crg);
    return r;
}
__device__ __forceinline__ float vgemm_slot_sum(const SlotRow& r, int nl) {
    const float* p = r.p + nl;
    float s = 0.f;
    int i = 0;
    for (; i + 8 <= r.ns; i += 8) {
        float t[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) t[j] = __ldcg(p + (size_t)(i + j) * 4096);
#pragma unroll
        for (int j = 0; j < 8; ++j) s += t[j];
    }
    for (; i < r.ns; ++i) s += __ldcg(p + (size_t)i * 4096);
    return s;
}
// Sum of slots for output (m, n), fixed slot order (deterministic). Loads are issued eight
// at a time before they are added, so a long slot list costs a few memory round trips
// rather than one per slot.
__device__ __forceinline__ float vgemm_part_get(const PartView& v, int m, int n) {
    const int crg = n >> 8, nl = n & 255;
    const int ns = vgemm_nslots(v, crg);
    const float* p = v.part + ((size_t)crg * v.max_slots * 16 + m) * 256 + nl;
    float s = 0.f;
    int i = 0;
    for (; i + 8 <= ns; i += 8) {
        float t[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) t[j] = __ldcg(p + (size_t)(i + j) * 16 * 256);
#pragma unroll
        for (int j = 0; j < 8; ++j) s += t[j];
    }
    for (; i < ns; ++i) s += __ldcg(p + (size_t)i * 16 * 256);
    return s;
}
// Four consecutive outputs n..n+3 (n % 4 == 0).
__device__ __forceinline__ float4 vgemm_part_get4(const PartView& v, int m, int n) {
    const int crg = n >> 8, nl = n & 255;
    const int ns = vgemm_nslots(v, crg);
    const float4* p = reinterpret_cast<const float4*>(v.part + ((size_t)crg * v.max_slots * 16 + m) * 256 + nl);
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    int i = 0;
    for (; i + 8 <= ns; i += 8) {
        float4 t[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) t[j] = __ldcg(p + (size_t)(i + j) * 16 * 64);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            s.x += t[j].x; s.y += t[j].y; s.z += t[j].z; s.w += t[j].w;
        }
    }
    for (; i < ns; ++i) {
        const float4 t = __ldcg(p + (size_t)i * 16 * 64);
        s.x += t.x; s.y += t.y; s.z += t.z; s.w += t.w;
    }
    return s;
}
#endif
