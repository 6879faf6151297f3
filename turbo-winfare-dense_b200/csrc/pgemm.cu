// Prefill GEMM: out[m][n] = sum_k (q[n][k] * s[n][k/64] + b[n][k/64]) * x[m][k] for a chunk
// of 17..128 prompt rows against INT4 G64 affine weights -- GemmInt4Batch
// (shaders/GemmInt4Batch.hlsl:64-143) on the sm_100a tcgen05 tensor cores. At M = 128 the
// INT4 stream is ~230 flop/B: the op is tensor-bound, where the verify GEMM (vgemm.cu) is
// HBM-bound, so this kernel is built around keeping the tensor pipe busy:
//   * one CTA per SM walks a contiguous stream-K range [c*T/C, (c+1)*T/C) of
//     (128-row tile, 64-group) units; a 4-stage shared-memory ring is filled by bulk copies
//     (cp.async.bulk, no multicast) completing on mbarriers: per unit the weight block
//     (4 KB of nibbles + 512 B of bf16 scale/bias) and the activation group's hi and lo
//     tiles, which the producing kernels wrote already in the MMA's 128-byte-swizzled
//     K-major image (common.cuh, wide layout);
//   * 4 converter warps turn each thread's weight row into 32 packed fp16x2 words -- nibble
//     q becomes the exact subnormal q * 2^-24 with one shift and one AND per pair (the
//     weights are stored pair-interleaved for this) -- and write them to tensor memory,
//     where they are the MMA's A operand;
//   * one thread issues tcgen05.mma kind::f16 (M = 128 weight rows, N = the chunk's rows
//     rounded up to 16, K = 16): 4 k-slices x {hi, lo} activation terms per group into a
//     double-buffered fp32 accumulator in tensor memory, and tcgen05.commit signals the
//     epilogue and frees the stage;
//   * 16 epilogue warps read the group's accumulator (tcgen05.ld) and apply the group's
//     scale and bias in fp32, acc += s * P + b * Y (products stay exact, each group is summed
//     in fp32); the activations' power-of-two scale is per row, so it is applied once, when
//     the tile segment is written;
//   * at the end of a tile segment the partial is written straight to the dense output when
//     one CTA covers the whole tile; otherwise to a fixed slot, and the last CTA to arrive
//     on the tile's counter adds the slots in slot order (deterministic).
// Every wait is bounded (2 s); a wait that gives up sets the error word and a CTA-wide abort
// flag, after which no wait blocks, so the CTA drains, frees its tensor memory and exits.
#include "common.cuh"
#include "launch.cuh"
#include "pgemm.h"
#include "tcgen05.cuh"
#include "tma.cuh"

#include <algorithm>

namespace g4b {
namespace {

// Ring depth measured against 3 and 5: a 31B 128-row pass takes 31.6 ms with 4, 32.5 with 5, 32.7 with 3.
constexpr int kStages = 4;
constexpr int kADepth = 4;  // A-operand buffers in tensor memory
constexpr int kConvWarps = 4;
constexpr int kEpiWarps = 16;
constexpr int kEpiCols = 128 / (kEpiWarps / 4);  // accumulator columns per epilogue warp
constexpr int kProdWarp = kConvWarps + kEpiWarps;  // 12
constexpr int kMmaWarp = kProdWarp + 1;            // 13
constexpr int kThreadsP = (kMmaWarp + 1) * 32;     // 448
// Each of the SM's four sub-partitions holds 16K registers for the warps scheduled on it.
constexpr int kMaxRegs = (512 / ((kThreadsP / 32 + 3) / 4)) / 8 * 8;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kAccCols = 128;          // one fp32 accumulator: 128 activation rows
constexpr int kAccBufs = 3;                 // accumulators in flight between MMA and epilogue
constexpr uint32_t kACol0 = kAccBufs * kAccCols;  // A buffers after the accumulators
constexpr uint32_t kACols = 32;             // 64 fp16 of a weight row
constexpr int kErrPgemm = 6;

// Stage layout (bytes): hi tile, lo tile, weight nibbles, scale/bias, the group's Y records.
constexpr uint32_t kOffHi = 0;
constexpr uint32_t kOffLo = kWideTileBytes;
constexpr uint32_t kOffW = 2 * kWideTileBytes;
constexpr uint32_t kOffSB = kOffW + 4096;
constexpr uint32_t kOffY = kOffSB + 512;
constexpr uint32_t kStageBytes = (kOffY + kPrefillRows * 4 + 1023) / 1024 * 1024;

struct Bars {
    uint64_t full[kStages], empty[kStages];
    uint64_t conv[kADepth], a_empty[kADepth];
    uint64_t acc_full[kAccBufs], acc_empty[kAccBufs];
    uint64_t done;
    uint32_t tmem_base;
    int abort;
    int last;
    // The CTA's first and last tiles may be shared with neighbouring CTAs (every tile in between
    // is wholly this CTA's): tile index, covering-CTA count and this CTA's slot for each.
    int seg_tile[2], seg_count[2], seg_slot[2];
};
constexpr size_t kSmemBytes = 1024 + kStages * kStageBytes + sizeof(Bars);

__device__ __forceinline__ long long cta_of_unit(long long u, long long T, int C) { return ((u + 1) * C - 1) / T; }

// Bounded wait that also returns (false) as soon as another warp of the CTA has given up.
__device__ __forceinline__ bool pg_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    while (!mbar_try_wait_sleep(bar, parity, 1000000u)) {
        if (*abort) return false;
        if (global_ns() - t0 > kWaitLimitNs) {
            *abort = 1;
            if (err) atomicExch(err, kErrPgemm);
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory"); }

__global__ void __maxnreg__(kMaxRegs) pgemm_kernel(PgemmParams p) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    Bars& bars = *reinterpret_cast<Bars*>(sm + kStages * kStageBytes);
    volatile int* abort = &bars.abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = p.K / 64;
    const long long T = (long long)p.n_tiles * G;
    const int C = gridDim.x, c = blockIdx.x;
    const long long u0 = (long long)c * T / C, u1 = (long long)(c + 1) * T / C;
    const int n = (int)(u1 - u0);
    const int nmma = min(kPrefillRows, (p.M + 15) & ~15);
    auto stage = [&](int s) { return sm + (size_t)s * kStageBytes; };

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&bars.full[s], 1);
            mbar_init(&bars.empty[s], kConvWarps + 1 + kEpiWarps);
        }
        for (int a = 0; a < kADepth; ++a) {
            mbar_init(&bars.conv[a], kConvWarps);
            mbar_init(&bars.a_empty[a], 1);
        }
        for (int b = 0; b < kAccBufs; ++b) {
            mbar_init(&bars.acc_full[b], 1);
            mbar_init(&bars.acc_empty[b], kEpiWarps);
        }
        mbar_init(&bars.done, 1);
        bars.abort = 0;
        for (int e = 0; e < 2; ++e) {
            const long long t = (e == 0 ? u0 : u1 - 1) / G;
            const long long cf = cta_of_unit(t * G, T, C), cl = cta_of_unit(t * G + G - 1, T, C);
            bars.seg_tile[e] = (int)t;
            bars.seg_count[e] = (int)(cl - cf + 1);
            bars.seg_slot[e] = (int)(c - cf);
        }
        mbar_init_fence();
    }
    if (warp == kMmaWarp) tc::alloc(&bars.tmem_base, kTmemCols);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = bars.tmem_base;
    pdl_launch_dependents();

    if (warp == kProdWarp) {
        // ---------------------------------------------------------------- producer
        if (lane == 0) {
            const char* wsrc = static_cast<const char*>(p.w);
            const char* hi = static_cast<const char*>(p.act);
            const char* lo = hi + (size_t)p.g_layout * kWideTileBytes;
            const char* ys = lo + (size_t)p.g_layout * kWideTileBytes;
            const uint32_t act_bytes = (uint32_t)nmma * 128, y_bytes = (uint32_t)nmma * 4;
            const uint32_t tx = kPgemmBlockBytes + 2 * act_bytes + y_bytes;
            auto copy_act = [&](int i) {
                const int s = i % kStages;
                const int g = (int)((u0 + i) % G);
                bulk_g2s(stage(s) + kOffHi, hi + (size_t)g * kWideTileBytes, act_bytes, &bars.full[s]);
                bulk_g2s(stage(s) + kOffLo, lo + (size_t)g * kWideTileBytes, act_bytes, &bars.full[s]);
                bulk_g2s(stage(s) + kOffY, ys + (size_t)g * kPrefillRows * 4, y_bytes, &bars.full[s]);
            };
            auto copy_w = [&](int i) {
                const int s = i % kStages;
                mbar_expect_tx(&bars.full[s], tx);
                bulk_g2s(stage(s) + kOffW, wsrc + (size_t)(u0 + i) * kPgemmBlockBytes, kPgemmBlockBytes,
                         &bars.full[s]);
            };
            // The weights do not depend on the previous kernel: start them before waiting.
            const int pre = min(n, kStages);
            for (int i = 0; i < pre; ++i) copy_w(i);
            pdl_wait();
            for (int i = 0; i < pre; ++i) copy_act(i);
            int issued = pre;
            for (int i = pre; i < n; ++i) {
                if (!pg_wait(&bars.empty[i % kStages], ((i / kStages) + 1) & 1, abort, p.err)) break;
                copy_w(i);
                copy_act(i);
                issued = i + 1;
            }
            // Let every issued copy land before the CTA can exit.
            for (int i = max(0, issued - kStages); i < issued; ++i)
                if (!mbar_wait(&bars.full[i % kStages], (i / kStages) & 1) && p.err) atomicExch(p.err, kErrPgemm);
        }
    } else if (warp == kMmaWarp) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            const uint32_t idesc = tc::idesc_f16(kPgemmTileRows, nmma);
            for (int i = 0; i < n; ++i) {
                const int s = i % kStages, a = i % kADepth, b = i % kAccBufs;
                bool ok = pg_wait(&bars.full[s], (i / kStages) & 1, abort, p.err);
                ok = ok && pg_wait(&bars.conv[a], (i / kADepth) & 1, abort, p.err);
                ok = ok && (i < kAccBufs || pg_wait(&bars.acc_empty[b], ((i / kAccBufs) + 1) & 1, abort, p.err));
                tc::fence_after_sync();
                if (ok) {
                    const uint32_t d = tmem + b * kAccCols;
                    const uint32_t at = tmem + kACol0 + a * kACols;
                    const uint32_t hs = smem_u32(stage(s) + kOffHi), ls = smem_u32(stage(s) + kOffLo);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        tc::mma_ts(d, at + kk * 8, tc::desc_sw128(hs + kk * 32), idesc, kk > 0 ? 1u : 0u);
                        tc::mma_ts(d, at + kk * 8, tc::desc_sw128(ls + kk * 32), idesc, 1u);
                    }
                }
                tc::commit(&bars.acc_full[b]);
                tc::commit(&bars.a_empty[a]);
                tc::commit(&bars.empty[s]);
            }
            // Every MMA has completed before tensor memory is freed.
            tc::commit(&bars.done);
            if (!mbar_wait(&bars.done, 0) && p.err) atomicExch(p.err, kErrPgemm);
        }
    } else if (warp < kConvWarps) {
        // ---------------------------------------------------------------- converters
        const int r = warp * 32 + lane;
        const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16) + kACol0;
        const int sw = (r >> 2) & 1;
        for (int i = 0; i < n; ++i) {
            const int s = i % kStages, a = i % kADepth;
            bool ok = pg_wait(&bars.full[s], (i / kStages) & 1, abort, p.err);
            ok = ok && (i < kADepth || pg_wait(&bars.a_empty[a], ((i / kADepth) + 1) & 1, abort, p.err));
            ok = __all_sync(0xffffffffu, ok);
            if (ok) {
                const unsigned char* wb = stage(s) + kOffW + r * 32;
                const uint4 h0 = *reinterpret_cast<const uint4*>(wb + (sw << 4));
                const uint4 h1 = *reinterpret_cast<const uint4*>(wb + ((sw ^ 1) << 4));
                const uint32_t words[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
                uint32_t v[32];
#pragma unroll
                for (int j = 0; j < 8; ++j)
#pragma unroll
                    for (int q = 0; q < 4; ++q) v[4 * j + q] = (words[j] >> (4 * q)) & 0x000F000Fu;
                tc::st32(trow + a * kACols, v);
                tc::wait_st();
            }
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&bars.conv[a]);
                mbar_arrive(&bars.empty[s]);
            }
        }
    } else {
        // ---------------------------------------------------------------- epilogue
        pdl_wait();  // the outputs and counters may still be read by the previous kernel
        const int q = warp & 3, part = (warp - kConvWarps) >> 2;
        const int r = q * 32 + lane;
        const int c0 = part * kEpiCols;
        const uint32_t tl = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0;
        float acc[kEpiCols];
#pragma unroll
        for (int j = 0; j < kEpiCols; ++j) acc[j] = 0.f;
        int t = (int)(u0 / G), g = (int)(u0 - (long long)t * G);  // unit u0 + i, advanced below
        for (int i = 0; i < n; ++i, g = (g + 1 == G) ? 0 : g + 1, t += (g == 0)) {
            const int s = i % kStages, b = i % kAccBufs;
            bool ok = pg_wait(&bars.acc_full[b], (i / kAccBufs) & 1, abort, p.err);
            ok = ok && pg_wait(&bars.full[s], (i / kStages) & 1, abort, p.err);
            ok = __all_sync(0xffffffffu, ok);
            tc::fence_after_sync();
            if (ok && c0 < nmma) {  // warp-uniform
                const uint32_t sbw = *reinterpret_cast<const uint32_t*>(stage(s) + kOffSB + r * 4);
                const float sc = bf16_lo(sbw), bi = bf16_hi(sbw);
                const float4* yv = reinterpret_cast<const float4*>(stage(s) + kOffY) + c0 / 4;
                // The rows' scales are per row, not per group: acc += s*P + b*Y here and the
                // row's E is applied once when the segment is written.
#pragma unroll
                for (int jc = 0; jc < kEpiCols; jc += 16) {
                    float P[16];
                    tc::ld16(tl + b * kAccCols + jc, P);
                    tc::wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; j += 4) {
                        const float4 y4 = yv[(jc + j) / 4];  // Y of columns jc+j .. jc+j+3
                        acc[jc + j] = fmaf(sc, P[j], fmaf(bi, y4.x, acc[jc + j]));
                        acc[jc + j + 1] = fmaf(sc, P[j + 1], fmaf(bi, y4.y, acc[jc + j + 1]));
                        acc[jc + j + 2] = fmaf(sc, P[j + 2], fmaf(bi, y4.z, acc[jc + j + 2]));
                        acc[jc + j + 3] = fmaf(sc, P[j + 3], fmaf(bi, y4.w, acc[jc + j + 3]));
                    }
                }
            }
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&bars.acc_empty[b]);
                mbar_arrive(&bars.empty[s]);
            }
            if (g != G - 1 && i != n - 1) continue;
            // ---- end of this CTA's segment of tile t
            const int row = t * kPgemmTileRows + r;
            const float* erow = reinterpret_cast<const float*>(static_cast<const char*>(p.act) +
                                                               2 * (size_t)p.g_layout * kWideTileBytes) +
                                (size_t)p.g_layout * kPrefillRows + c0;
            const int e = t == bars.seg_tile[0] ? 0 : 1;
            const int count = (t == bars.seg_tile[0] || t == bars.seg_tile[1]) ? bars.seg_count[e] : 1;
            if (count == 1) {
                if (row < p.N) {
                    float* yp = p.y + (size_t)c0 * p.ldy + row;
#pragma unroll
                    for (int j = 0; j < kEpiCols; ++j, yp += p.ldy)
                        if (c0 + j < p.M) *yp = acc[j] * (__ldg(erow + j) * 16777216.0f);
                }
            } else {
                // Every CTA of the tile writes its slot; the last to arrive re-reads all of them
                // (64 independent loads per slot in flight) and adds them in slot order.
                const int slot = bars.seg_slot[e];
                float* base = p.part + (size_t)t * p.max_slots * (kPgemmTileRows * 128) + (size_t)c0 * 128 + r;
                {
                    float* sp = base + (size_t)slot * (kPgemmTileRows * 128);
#pragma unroll
                    for (int j = 0; j < kEpiCols; ++j) __stcg(sp + j * 128, acc[j]);
                }
                __threadfence();
                epi_bar();
                if (warp == kConvWarps && lane == 0) {
                    const unsigned old = atomicAdd(&p.cnt[t], 1u);
                    bars.last = old == (unsigned)(count - 1);
                }
                epi_bar();
                if (bars.last) {
                    __threadfence();
#pragma unroll
                    for (int j = 0; j < kEpiCols; ++j) acc[j] = 0.f;
                    for (int sl = 0; sl < count; ++sl) {
                        const float* sp = base + (size_t)sl * (kPgemmTileRows * 128);
#pragma unroll
                        for (int jc = 0; jc < kEpiCols; jc += 8) {
                            float v[8];
#pragma unroll
                            for (int j = 0; j < 8; ++j) v[j] = __ldcg(sp + (jc + j) * 128);
#pragma unroll
                            for (int j = 0; j < 8; ++j) acc[jc + j] += v[j];
                        }
                    }
                    if (row < p.N) {
                        float* yp = p.y + (size_t)c0 * p.ldy + row;
#pragma unroll
                        for (int j = 0; j < kEpiCols; ++j, yp += p.ldy)
                            if (c0 + j < p.M) *yp = acc[j] * (__ldg(erow + j) * 16777216.0f);
                    }
                    if (warp == kConvWarps && lane == 0) p.cnt[t] = 0;
                }
            }
#pragma unroll
            for (int j = 0; j < kEpiCols; ++j) acc[j] = 0.f;
        }
    }

    tc::fence_before_sync();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc::fence_after_sync();
        tc::dealloc(tmem, kTmemCols);
    }
}

// Container word (nibble j = k 8w+j at bits 4j) -> pair-interleaved word: positions 0..3 hold
// the even k (0,2,4,6), positions 4..7 the odd k, so (word >> 4p) & 0x000F000F is the fp16x2
// pair (k 2p, k 2p+1).
__device__ __forceinline__ uint32_t pair_interleave(uint32_t w) {
    uint32_t o = 0;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        o |= ((w >> (8 * p)) & 0xFu) << (4 * p);
        o |= ((w >> (8 * p + 4)) & 0xFu) << (16 + 4 * p);
    }
    return o;
}

// One thread per (tile, group, row): 32 bytes of nibbles (the two 16-byte halves swapped on
// rows with bit 2 set, so the converter warps' 16-byte loads are bank-conflict free) and the
// row's scale/bias word.
__global__ void pgemm_repack_kernel(const uint32_t* __restrict__ W, const uint16_t* __restrict__ S,
                                    const uint16_t* __restrict__ B, int N, int K, int n_tiles,
                                    unsigned char* __restrict__ out) {
    const int G = K / 64, wpr = K / 8;
    const long long total = (long long)n_tiles * G * kPgemmTileRows;
    for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
         idx += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(idx % kPgemmTileRows);
        const long long tg = idx / kPgemmTileRows;
        const int g = (int)(tg % G);
        const long long t = tg / G;
        const long long row = t * kPgemmTileRows + r;
        uint32_t v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = row < N ? pair_interleave(W[row * wpr + g * 8 + j]) : 0u;
        unsigned char* blk = out + (size_t)tg * kPgemmBlockBytes;
        const int sw = (r >> 2) & 1;
        *reinterpret_cast<uint4*>(blk + r * 32 + (sw << 4)) = make_uint4(v[0], v[1], v[2], v[3]);
        *reinterpret_cast<uint4*>(blk + r * 32 + ((sw ^ 1) << 4)) = make_uint4(v[4], v[5], v[6], v[7]);
        uint32_t sb = 0;
        if (row < N) sb = (uint32_t)S[row * G + g] | ((uint32_t)B[row * G + g] << 16);
        *reinterpret_cast<uint32_t*>(blk + 4096 + r * 4) = sb;
    }
}

}  // namespace
}  // namespace g4b

using namespace g4b;

int pgemm_grid(int n_tiles, int groups) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long long T = (long long)n_tiles * groups;
    return (int)std::max<long long>(1, std::min<long long>(sms, T));
}

int pgemm_max_slots(int n_tiles, int groups, int grid) {
    const long long T = (long long)n_tiles * groups;
    int mx = 1;
    for (int t = 0; t < n_tiles; ++t) {
        const long long a = ((long long)t * groups + 1) * grid - 1, b = ((long long)(t + 1) * groups) * grid - 1;
        mx = std::max(mx, (int)(b / T - a / T + 1));
    }
    return mx;
}

cudaError_t pgemm_repack(const uint32_t* W, const uint16_t* S, const uint16_t* B, int N, int K, void* out,
                         cudaStream_t st) {
    if (N <= 0 || K <= 0 || K % 64) return cudaErrorInvalidValue;
    pgemm_repack_kernel<<<1184, 256, 0, st>>>(W, S, B, N, K, pgemm_n_tiles(N), static_cast<unsigned char*>(out));
    return cudaGetLastError();
}

cudaError_t pgemm_launch(const PgemmParams& p, cudaStream_t st, bool pdl) {
    if (!p.w || !p.act || !p.y || !p.part || !p.cnt || p.K <= 0 || p.K % 64 || p.M < 1 || p.M > kPrefillRows ||
        p.N <= 0 || p.n_tiles != pgemm_n_tiles(p.N) || p.ldy < p.N || p.g_layout < p.K / 64)
        return cudaErrorInvalidValue;
    const int grid = pgemm_grid(p.n_tiles, p.K / 64);
    if (pgemm_max_slots(p.n_tiles, p.K / 64, grid) > p.max_slots) return cudaErrorInvalidValue;
    static bool attr_set = false;
    if (!attr_set) {
        const cudaError_t e =
            cudaFuncSetAttribute(pgemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    return launch(pgemm_kernel, dim3(grid), dim3(kThreadsP), kSmemBytes, st, pdl, p);
}
