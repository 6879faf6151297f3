// Shared device-side definitions for the B200 speculative-decode kernels (sm_100a).
//
// Data formats in HBM (all fully resident):
//
// 1. Packed INT4 G64 weight matrix ("vgemm layout"), repacked once at load from the
//    container's row-major form (W [N][K/8] u32, scales/biases [N][K/64] bf16;
//    src/cpu_reference.cpp:367-381). Rows are grouped in warp row groups of 64 rows
//    (four 16-row MMA tiles) and K in 128-column k-tiles. Each (row group, k-tile) is one
//    contiguous 4608-byte block:
//      [r 0..3][half 0..1][lane 0..31] uint4   nibble words, 4096 B
//      [r 0..3][g 0..7] uint4                  bf16 scale/bias pairs, 512 B
//    Lane (g = lane/4, t = lane%4) of half h holds the words of rows g and g+8 covering
//    k = 32*kk + 8t .. +7 for kk = 2h and 2h+1, in the order {row g kk=2h, row g+8 kk=2h,
//    row g kk=2h+1, row g+8 kk=2h+1}: exactly the A-fragment words that lane needs for
//    mma.m16n8k16, so one 128-bit load per half feeds eight MMAs with no shuffles.
//    The scale/bias uint4 for (r, g) is {s(g,G0)|b(g,G0)<<16, s(g+8,G0)|b(g+8,G0)<<16,
//    s(g,G1)|b(g,G1)<<16, s(g+8,G1)|b(g+8,G1)<<16} for the two 64-groups G0, G1 of the
//    k-tile. Blocks are ordered [row group][k-tile], so a warp streams one row group's
//    k-range from contiguous memory. Rows beyond N and columns beyond K are zero.
//
// 2. Activation fragments ("B-frag layout") for the verify GEMM's B operand. An activation
//    matrix x [M][K] (M <= 16 verify/prefill rows) is stored as fp16 hi/lo pairs of
//    x / E, where E is a power of two chosen per (64-group, row) so |x/E| < 2^11:
//      frag[K/32][NB][32 lanes] uint4, gsum[K/64][NACC][8 cols] float2 {E, Y}
//    NB/NACC depend on M (see BMode). Y = 2^-24 * sum of the group's (hi+lo) values;
//    the per-group epilogue adds E*(s*P + b*Y), which restates q*s+b dequantization
//    exactly: sum_k (q s + b) x = s * sum q x + b * sum x.
//
// 3. INT4 nibbles enter the tensor core as IEEE fp16 SUBNORMALS: the bit pattern q (or
//    16q for odd nibbles) is the value q * 2^-24, so a single AND turns two nibbles into
//    an exact fp16x2 operand; the 2^24 (and 1/16) factors are folded into the activation
//    fragments and the final scale.
//    M = 5..16 use format 5 below instead.
//
// 5. Integer digits (verify rows 5..16). Per (64-group, row) a power-of-two E puts the group's
//    values on a 23-bit signed grid, v = rint(x / E) with |v| < 2^22, split into balanced
//    base-256 digits v = d0 + 256 d1 + 65536 d2 (each in [-128, 127]). Digit d of row m is MMA
//    column digit_col(m, d). For the k32 step kk, lane (g, t) of n-tile nt holds
//      b0 = bytes i = 0..3 of column g at k = 32 kk + 8t + 2i, b1 = the same at k + 1
//    which matches the A fragments the weight words give with two ANDs (even nibbles, odd
//    nibbles). frag[K/32][nt][32 lanes] uint2, gsum[K/64][16 rows] float2 {E, Y = sum v}.
//    The MMA sums q * d exactly in int32; the epilogue forms P = sum q v in fp32 and adds
//    E * (s * P + b * Y).
//
// 4. Wide activation layout, for passes of 17..128 rows (prefill chunks) feeding the
//    tcgen05 prefill GEMM (pgemm.cu). The same fp16 hi/lo split, but with ONE power-of-two
//    scale E per row (|x/E| < 2^11 for the row's largest element), so the GEMM can add the
//    groups' scaled sums and apply E once per output. Stored as ready-made shared-memory images
//    of the MMA's B operand: per 64-group g, a 16 KB hi tile and a 16 KB lo tile of 128 rows x
//    64 fp16 in the 128-byte-swizzled K-major form (row m at byte m*128, 16-byte chunk c of the
//    row at chunk position c ^ (m % 8)), then the groups' Y records and the rows' scales:
//      hi[K/64][16384 B], lo[K/64][16384 B], ysum[K/64][128 rows] float, erow[128] float
//    so one bulk copy per tile lands it in shared memory exactly as the MMA reads it.
#pragma once
#include <cuda_fp16.h>
#include <cstdint>

#include "passrows.h"

namespace g4b {

constexpr int kRowsPerTile = 16;         // MMA M
constexpr int kTilesPerWarp = 4;         // row tiles per warp
constexpr int kWarpRows = kRowsPerTile * kTilesPerWarp;  // 64
constexpr int kKTile = 128;              // k-tile width
constexpr int kKTileBytes = 4608;        // one (row group, k-tile) block
constexpr int kNibBytes = 4096;
constexpr int kWideTileBytes = kPrefillRows * 128;  // one 64-group's hi (or lo) tile

// B-operand mode for M rows. M <= 4 packs the fp16 hi and lo terms of every row into one
// m16n8k16 tile. M = 5..16 uses integer digits instead (format 5): three signed 8-bit digits
// per value, multiplied by the nibbles with mma.sync m16n8k32 (u8 x s8 -> s32), which does
// twice the work per instruction of the fp16 MMA at the same issue rate on sm_100a.
struct BMode {
    int nb;      // fp16 modes: B tiles per k32 block
    int nacc;    // fp16 modes: accumulator column tiles
    bool packed; // M <= 4: hi in columns 0..3, lo in columns 4..7 of one tile
    int nt;      // digit modes: n-tiles of 8 digit columns (0 = fp16 mode)
};
__host__ __device__ inline BMode bmode_for(int M) {
    if (M <= 4) return {1, 1, true, 0};
    if (M <= 5) return {0, 0, false, 2};
    if (M <= 8) return {0, 0, false, 3};
    if (M <= 10) return {0, 0, false, 4};
    return {0, 0, false, 6};
}
__host__ __device__ inline size_t bfrag_frag_bytes(int K, int M) {
    const BMode md = bmode_for(M);
    return md.nt ? (size_t)(K / 32) * md.nt * 32 * 8 : (size_t)(K / 32) * md.nb * 512;
}
__host__ __device__ inline size_t bfrag_gsum_bytes(int K, int M) {
    const BMode md = bmode_for(M);
    return (size_t)(K / 64) * (md.nt ? kMaxM : md.nacc * 8) * sizeof(float2);
}
// Digit modes: the (n-tile, column) of digit d of activation row m. Columns are arranged so
// that the quad thread t holding accumulator columns 2t, 2t+1 holds all three digits of rows
// t, 4+t (and 8+t, 12+t with six tiles); with two tiles, row 4's digits sit in column 2d+1 of
// tile 1 (threads 0..2) and are gathered with two shuffles; with four tiles (9..10 rows), rows
// 8 and 9 sit in columns 2d and 2d+1 of tile 3 and are gathered the same way.
__host__ __device__ inline void digit_col(int nt_count, int m, int d, int& nt, int& col) {
    if (nt_count == 2 && m == 4) {
        nt = 1;
        col = 2 * d + 1;
        return;
    }
    if (nt_count == 4 && m >= 8) {  // rows 8 and 9: tile 3, columns 2d (row 8) and 2d+1 (row 9)
        nt = 3;
        col = 2 * d + (m - 8);
        return;
    }
    const int blk = m >> 3, mm = m & 7, tt = mm & 3;
    if (mm < 4) {
        nt = 3 * blk + (d < 2 ? 0 : 1);
        col = d < 2 ? 2 * tt + d : 2 * tt;
    } else {
        nt = 3 * blk + (d == 0 ? 1 : 2);
        col = d == 0 ? 2 * tt + 1 : 2 * tt + (d - 1);
    }
}
// Bytes of the wide layout (M > kMaxM) for K columns.
__host__ __device__ inline size_t wide_bytes(int K) {
    return (size_t)(K / 64) * (2 * kWideTileBytes + kPrefillRows * sizeof(float)) + kPrefillRows * sizeof(float);
}
// Capacity of one activation buffer for K columns at any M (either layout).
__host__ __device__ inline size_t bfrag_capacity(int K) {
    const size_t narrow = bfrag_frag_bytes(K, kMaxM) + bfrag_gsum_bytes(K, kMaxM);
    const size_t wide = wide_bytes(K);
    return narrow > wide ? narrow : wide;
}

struct BFragView {
    uint4* frag;      // B-frag layout: [K/32][nb][32];  wide layout: the hi tiles
    float2* gsum;     // B-frag layout: [K/64][nacc][8] {E, Y}
    uint32_t lo_off;  // wide layout: bytes from a group's hi tile to its lo tile; 0 = B-frag layout
    float* ysum;      // wide layout: [K/64][128] Y records
    float* erow;      // wide layout: [128] row scales E
};
__host__ __device__ inline BFragView bfrag_view(void* base, int K, int M) {
    BFragView v;
    v.frag = reinterpret_cast<uint4*>(base);
    if (M > kMaxM) {
        v.lo_off = (uint32_t)((K / 64) * kWideTileBytes);
        v.gsum = nullptr;
        v.ysum = reinterpret_cast<float*>(reinterpret_cast<char*>(base) + 2 * (size_t)v.lo_off);
        v.erow = v.ysum + (size_t)(K / 64) * kPrefillRows;
    } else {
        v.lo_off = 0;
        v.gsum = reinterpret_cast<float2*>(reinterpret_cast<char*>(base) + bfrag_frag_bytes(K, M));
        v.ysum = v.erow = nullptr;
    }
    return v;
}
// Row scale of the wide layout for a row whose largest |x| is amax (a power of two, so the
// scaled row stays below 2^11 and the hi/lo split is exact to ~2^-22 of amax).
__device__ __forceinline__ float wide_row_scale(float amax) {
    int e = 0;
    frexpf(amax, &e);
    return amax > 0.f ? ldexpf(1.0f, e - 11) : 1.0f;
}

__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }
__device__ __forceinline__ float bf16_to_f32(uint16_t v) { return __uint_as_float((uint32_t)v << 16); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ int warp_sum_int(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide sum for blockDim.x <= 1024; `red` needs 32 floats of shared memory.
// Two block-wide sums in one exchange: each warp's partials are added in warp order by every
// thread. `red` (32 entries) must not be written again by the block without a barrier first.
__device__ __forceinline__ float2 block_sum2(float2 v, float2* red) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    v.x = warp_sum(v.x);
    v.y = warp_sum(v.y);
    if (lane == 0) red[wid] = v;
    __syncthreads();
    const int nw = (blockDim.x + 31) >> 5;
    float2 t = red[0];
    for (int i = 1; i < nw; ++i) {
        t.x += red[i].x;
        t.y += red[i].y;
    }
    return t;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    const int nw = (blockDim.x + 31) >> 5;
    float t = (threadIdx.x < nw) ? red[threadIdx.x] : 0.0f;
    if (wid == 0) t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
    __syncthreads();
    const float r = red[0];
    __syncthreads();
    return r;
}

// Block-wide max of non-negative values for blockDim.x <= 1024; `red` needs 32 floats.
__device__ __forceinline__ float block_max(float v, float* red) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    const int nw = (blockDim.x + 31) >> 5;
    float t = (threadIdx.x < nw) ? red[threadIdx.x] : 0.0f;
    if (wid == 0) t = warp_max(t);
    if (threadIdx.x == 0) red[0] = t;
    __syncthreads();
    const float r = red[0];
    __syncthreads();
    return r;
}

// Programmatic dependent launch: wait for the producing kernel's writes / let the next
// kernel start its independent prologue (weight prefetch) early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// Kernel entry under PDL: let the next kernel in the stream launch now (it only runs its
// own prologue until it waits in turn), then wait for this kernel's producer to finish.
// Every kernel calls this before touching anything a predecessor wrote.
__device__ __forceinline__ void pdl_enter() {
    pdl_launch_dependents();
    pdl_wait();
}

}  // namespace g4b
