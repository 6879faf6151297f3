// Verify GEMM: out[m][n] = sum_k (q[n][k] * s[n][k/64] + b[n][k/64]) * x[m][k] for M <= 16
// rows against INT4 G64 affine weights -- GemmInt4Batch / GemvInt4
// (shaders/GemmInt4Batch.hlsl:64-143, shaders/Common.hlsli:163-222) rebuilt for sm_100a.
//
// The op is HBM-bound (0.5625 B per weight; 3.5-56 flop/B for M = 1..16), so the kernel is
// organised around streaming the packed weights once at full bandwidth:
//   * weights stream in the vgemm layout (common.cuh) with 128-bit non-allocating loads,
//     one k-tile ahead in registers, so every warp keeps 4.5 KB in flight;
//   * nibbles become exact fp16-subnormal tensor-core operands with one AND each, and
//     mma.sync m16n8k16 (fp32 accumulate) does the multiply-adds -- the activations ride as
//     fp16 hi/lo pairs, which keeps fp32-level accuracy (|error| ~ 2^-22 relative) where a
//     bf16 dequantisation would give ~2^-9;
//   * scale and bias are applied per 64-group in fp32 from the group partial sums;
//   * work is split stream-K style: CTA c owns a contiguous range of (row group, k-tile)
//     units, so every CTA streams the same number of bytes whatever the shape. Row groups
//     split across CTAs are reduced deterministically (fixed slot order) by the last CTA
//     to finish, which also resets the group's arrival counter for the next launch.
// tcgen05 is deliberately not used here: at M <= 16 the tensor work is a few percent of the
// issue budget and the binding resource is HBM bandwidth.
#include "common.cuh"
#include "vgemm.h"

#include <algorithm>
#include <cuda_runtime.h>

namespace g4b {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kCtaRows = kWarps * kWarpRows;  // 256
constexpr int kBChunk = 8;                    // k-tiles of B fragments staged at a time

__device__ __forceinline__ uint4 ldg_stream(const uint4* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ void mma16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1, const float* c) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]),
          "f"(c[3]));
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

struct KTileRegs {
    uint4 nib[kTilesPerWarp][2];
    uint4 sb[kTilesPerWarp];
};

__device__ __forceinline__ void load_ktile(KTileRegs& R, const uint4* blk, int lane) {
#pragma unroll
    for (int r = 0; r < kTilesPerWarp; ++r) {
        R.nib[r][0] = ldg_stream(blk + (r * 2 + 0) * 32 + lane);
        R.nib[r][1] = ldg_stream(blk + (r * 2 + 1) * 32 + lane);
    }
#pragma unroll
    for (int r = 0; r < kTilesPerWarp; ++r) R.sb[r] = ldg_stream(blk + 256 + r * 8 + (lane >> 2));
}

// One k-tile for one warp: 4 row tiles x 128 k. P = group partials, acc = totals.
template <int NB, int NACC, bool PACKED>
__device__ __forceinline__ void compute_ktile(const KTileRegs& R, const uint4* bsm, const float4* gsm,
                                              float (&acc)[kTilesPerWarp][NACC][4], int lane) {
    constexpr uint32_t M0 = 0x000F000Fu, M1 = 0x00F000F0u;
    const float zero[4] = {0.f, 0.f, 0.f, 0.f};
    float P[kTilesPerWarp][NACC][4];
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
        uint4 bf[NB];
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) bf[nb] = bsm[(kk * NB + nb) * 32 + lane];
        const bool first = (kk & 1) == 0;
#pragma unroll
        for (int r = 0; r < kTilesPerWarp; ++r) {
            const uint4& h = R.nib[r][kk >> 1];
            const uint32_t wg = (kk & 1) ? h.z : h.x;
            const uint32_t wg8 = (kk & 1) ? h.w : h.y;
            const uint32_t wg2 = wg >> 8, wg82 = wg8 >> 8;
#pragma unroll
            for (int a = 0; a < NACC; ++a) {
                // step A: k slots {0,4} and 16x{1,5}
                mma16816(P[r][a], wg & M0, wg8 & M0, wg & M1, wg8 & M1, bf[PACKED ? 0 : 2 * a].x,
                         bf[PACKED ? 0 : 2 * a].y, first ? zero : P[r][a]);
                if (!PACKED)
                    mma16816(P[r][a], wg & M0, wg8 & M0, wg & M1, wg8 & M1, bf[2 * a + 1].x,
                             bf[2 * a + 1].y, P[r][a]);
                // step B: k slots {2,6} and 16x{3,7}
                mma16816(P[r][a], wg2 & M0, wg82 & M0, wg2 & M1, wg82 & M1, bf[PACKED ? 0 : 2 * a].z,
                         bf[PACKED ? 0 : 2 * a].w, P[r][a]);
                if (!PACKED)
                    mma16816(P[r][a], wg2 & M0, wg82 & M0, wg2 & M1, wg82 & M1, bf[2 * a + 1].z,
                             bf[2 * a + 1].w, P[r][a]);
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
                    const uint32_t sbg = G ? R.sb[r].z : R.sb[r].x;
                    const uint32_t sbg8 = G ? R.sb[r].w : R.sb[r].y;
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

// First CTA whose unit range contains unit x (ranges are floor(c*T/G) .. floor((c+1)*T/G)).
__device__ __forceinline__ long long cta_of_unit(long long x, long long T, long long G) {
    return ((x + 1) * G + T - 1) / T - 1;
}

// Stages the B fragments and {E, Y} records of k-tiles [kt, kt + kBChunk) into shared
// memory when kt starts a chunk. Called uniformly by every warp of the CTA.
template <int NB, int NACC>
__device__ __forceinline__ void stage_bfrags(const VgemmParams& p, uint4* bsm, float4* gsm, int kt,
                                             int kt0, int kt1) {
    if ((kt - kt0) % kBChunk != 0) return;
    const int ce = min(kt1, kt + kBChunk);
    __syncthreads();
    const int nf = (ce - kt) * 4 * NB * 32;  // uint4 count
    const uint4* fsrc = p.bfrag + (size_t)kt * 4 * NB * 32;
    for (int i = threadIdx.x; i < nf; i += kThreads) cp_async16(bsm + i, fsrc + i);
    const int ng = (ce - kt) * 2 * NACC * 4;  // float4 count
    const float4* gsrc = reinterpret_cast<const float4*>(p.gsum) + (size_t)kt * 2 * NACC * 4;
    for (int i = threadIdx.x; i < ng; i += kThreads) cp_async16(gsm + i, gsrc + i);
    cp_async_wait_all();
    __syncthreads();
}

template <int NB, int NACC, bool PACKED>
__global__ void __launch_bounds__(kThreads, NACC == 2 ? 2 : 3) vgemm_kernel(VgemmParams p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    uint4* bsm = reinterpret_cast<uint4*>(smem_raw);  // [kBChunk*4][NB][32]
    float4* gsm = reinterpret_cast<float4*>(smem_raw + kBChunk * 4 * NB * 512);  // [kBChunk*2][NACC][4]
    __shared__ int s_last;

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const long long T = (long long)p.n_crg * p.ktiles;
    const long long G = gridDim.x;
    const long long c = blockIdx.x;
    long long u = c * T / G;
    const long long u_end = (c + 1) * T / G;
    const uint4* wbase = reinterpret_cast<const uint4*>(p.w);

    bool waited = false;
    while (u < u_end) {
        const int crg = (int)(u / p.ktiles);
        const int kt0 = (int)(u % p.ktiles);
        const int kt1 = (int)min((long long)p.ktiles, (long long)kt0 + (u_end - u));
        const int wrg = crg * kWarps + warp;
        const bool active = wrg < p.n_wrg;
        const uint4* wrow = wbase + ((size_t)wrg * p.ktiles) * (kKTileBytes / 16);

        float acc[kTilesPerWarp][NACC][4];
#pragma unroll
        for (int r = 0; r < kTilesPerWarp; ++r)
#pragma unroll
            for (int a = 0; a < NACC; ++a)
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[r][a][i] = 0.f;

        KTileRegs ra, rb;
        if (active) load_ktile(ra, wrow + (size_t)kt0 * (kKTileBytes / 16), lane);
        if (!waited) {
            // Weights do not depend on the previous kernel; activations and outputs do.
            pdl_wait();
            waited = true;
        }
        // Two k-tiles per trip so the double buffer never needs register copies. kBChunk is
        // even, so chunk boundaries only fall on the first half of a trip.
        for (int kt = kt0; kt < kt1; kt += 2) {
            stage_bfrags<NB, NACC>(p, bsm, gsm, kt, kt0, kt1);
            const int ci = (kt - kt0) % kBChunk;
            if (active) {
                if (kt + 1 < kt1) load_ktile(rb, wrow + (size_t)(kt + 1) * (kKTileBytes / 16), lane);
                compute_ktile<NB, NACC, PACKED>(ra, bsm + ci * 4 * NB * 32, gsm + ci * 2 * NACC * 4, acc, lane);
            }
            if (kt + 1 >= kt1) break;
            if (active) {
                if (kt + 2 < kt1) load_ktile(ra, wrow + (size_t)(kt + 2) * (kKTileBytes / 16), lane);
                compute_ktile<NB, NACC, PACKED>(rb, bsm + (ci + 1) * 4 * NB * 32, gsm + (ci + 1) * 2 * NACC * 4, acc, lane);
            }
        }

        // ---- segment epilogue ----
        const bool full = (kt0 == 0 && kt1 == p.ktiles);
        const float kScale = 16777216.0f;  // 2^24
        const int g = lane >> 2, t = lane & 3;
        int slot = 0, nslots = 1;
        if (!full) {
            const long long lo = cta_of_unit((long long)crg * p.ktiles, T, G);
            const long long hi = cta_of_unit((long long)(crg + 1) * p.ktiles - 1, T, G);
            slot = (int)(c - lo);
            nslots = (int)(hi - lo + 1);
        }
        if (active) {
#pragma unroll
            for (int r = 0; r < kTilesPerWarp; ++r) {
#pragma unroll
                for (int a = 0; a < NACC; ++a) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        float v = acc[r][a][i];
                        if (PACKED) v += __shfl_xor_sync(0xffffffffu, v, 2);
                        acc[r][a][i] = v * kScale;
                    }
                    if (PACKED && t >= 2) continue;
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int m = a * 8 + 2 * t + (i & 1);
                        const int nl = warp * kWarpRows + r * 16 + g + ((i >> 1) << 3);
                        const int n = crg * kCtaRows + nl;
                        if (m >= p.M) continue;
                        if (full) {
                            if (n < p.N) p.out[(size_t)m * p.ldo + n] = acc[r][a][i];
                        } else {
                            p.part[(((size_t)crg * p.max_slots + slot) * kMaxM + m) * kCtaRows + nl] = acc[r][a][i];
                        }
                    }
                }
            }
        }
        if (!full) {
            __threadfence();
            __syncthreads();
            if (threadIdx.x == 0) {
                const int prev = atomicAdd(p.counters + crg, 1);
                s_last = (prev == nslots - 1);
            }
            __syncthreads();
            if (s_last) {
                __threadfence();
                const float* base = p.part + (size_t)crg * p.max_slots * kMaxM * kCtaRows;
                for (int i = threadIdx.x; i < p.M * kCtaRows; i += kThreads) {
                    const int m = i / kCtaRows, nl = i % kCtaRows;
                    const int n = crg * kCtaRows + nl;
                    float s = 0.f;
                    for (int sl = 0; sl < nslots; ++sl)
                        s += __ldcg(base + ((size_t)sl * kMaxM + m) * kCtaRows + nl);
                    if (n < p.N) p.out[(size_t)m * p.ldo + n] = s;
                }
                if (threadIdx.x == 0) p.counters[crg] = 0;
            }
        }
        u += (kt1 - kt0);
    }
    if (!waited) pdl_wait();
}

template <int NB, int NACC, bool PACKED>
static size_t smem_bytes() {
    return (size_t)kBChunk * 4 * NB * 512 + (size_t)kBChunk * 2 * NACC * 4 * sizeof(float4);
}

template <int NB, int NACC, bool PACKED>
static int max_ctas_per_sm() {
    static int cached = -1;
    if (cached < 0) {
        const size_t sm = smem_bytes<NB, NACC, PACKED>();
        cudaFuncSetAttribute(vgemm_kernel<NB, NACC, PACKED>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        int n = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, vgemm_kernel<NB, NACC, PACKED>, kThreads, sm);
        cached = n > 0 ? n : 1;
    }
    return cached;
}

static int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    }
    return n;
}

template <int NB, int NACC, bool PACKED>
static cudaError_t launch_t(VgemmParams p, int grid, cudaStream_t st, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem_bytes<NB, NACC, PACKED>();
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, vgemm_kernel<NB, NACC, PACKED>, p);
}

}  // namespace g4b

using namespace g4b;

int vgemm_grid(int M, int n_crg, int ktiles) {
    const BMode md = bmode_for(M);
    int per_sm;
    if (md.packed) per_sm = max_ctas_per_sm<1, 1, true>();
    else if (md.nb == 2) per_sm = max_ctas_per_sm<2, 1, false>();
    else per_sm = max_ctas_per_sm<4, 2, false>();
    const long long T = (long long)n_crg * ktiles;
    return (int)std::min<long long>(T, (long long)sm_count() * per_sm);
}

int vgemm_max_slots(int grid, int n_crg, int ktiles) {
    // Every CTA owns at least floor(T/G) units, so a row group's `ktiles` units meet at most
    // ceil(ktiles / floor(T/G)) + 1 CTA ranges.
    const long long T = (long long)n_crg * ktiles;
    const long long min_units = std::max<long long>(1, T / grid);
    return (int)((ktiles + min_units - 1) / min_units + 1);
}

cudaError_t vgemm_launch(const VgemmParams& p, int grid, cudaStream_t st, bool pdl) {
    if (p.M < 1 || p.M > kMaxM) return cudaErrorInvalidValue;
    const BMode md = bmode_for(p.M);
    if (md.packed) return launch_t<1, 1, true>(p, grid, st, pdl);
    if (md.nb == 2) return launch_t<2, 1, false>(p, grid, st, pdl);
    return launch_t<4, 2, false>(p, grid, st, pdl);
}
