// Verify GEMM: out[m][n] = sum_k (q[n][k] * s[n][k/64] + b[n][k/64]) * x[m][k] for M <= 16
// rows against INT4 G64 affine weights -- GemmInt4Batch / GemvInt4
// (shaders/GemmInt4Batch.hlsl:64-143, shaders/Common.hlsli:163-222) rebuilt for sm_100a.
//
// The op is HBM-bound (0.5625 B per weight; 3.5-56 flop/B for M = 1..16), so the kernel is
// organised around streaming the packed weights once at full bandwidth:
//   * each warp owns a 2- or 4-stage ring of 4608-byte k-tile blocks in shared memory, filled by
//     TMA bulk copies (cp.async.bulk, one per block, completion on a per-stage mbarrier).
//     The first stages are issued before griddepcontrol.wait, so under programmatic
//     dependent launch the weight stream starts while the previous kernel is still draining;
//   * nibbles become exact fp16-subnormal tensor-core operands with one AND each, and
//     mma.sync m16n8k16 (fp32 accumulate) does the multiply-adds; the activations ride as
//     fp16 hi/lo pairs (B-frag layout, common.cuh), keeping fp32-level accuracy;
//   * scale and bias are applied per 64-group in fp32 from the group partial sums;
//   * work is split stream-K style: CTA c owns the contiguous unit range
//     [c*T/G, (c+1)*T/G) of (256-row group, k-tile) units, so every CTA streams the same
//     number of bytes whatever the shape. Each CTA writes one partial per row group it
//     touches into a fixed slot; the last CTA to arrive on a row group adds its slots in
//     slot order (deterministic) and writes the dense output;
//   * activation fragments for the CTA's k-range are double-buffered in shared memory by
//     bulk copies, one chunk ahead.
// tcgen05 is deliberately not used here: at M <= 16 the tensor work is a small part of the
// issue budget and the binding resource is HBM bandwidth.
#include "common.cuh"
#include "launch.cuh"
#include "tma.cuh"
#include "vgemm.h"
#include "vgemm_tile.cuh"

#include <algorithm>
#include <cuda_runtime.h>

namespace g4b {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kCtaRows = kWarps * kWarpRows;  // 256
// Weight ring depth per warp, by mode, as measured against 3 stages: the packed fp16 mode
// (1..4 rows: the drafter's one-row steps, a few units per CTA) gains from the deeper prefetch
// before the PDL wait (E2B drafter step 1.411 -> 1.377 ms with 4 stages); the 5..8-row digit
// modes run faster with fewer weight bytes in flight ahead of each CTA (31B 5-row verify pass
// 6.07 -> 5.84 ms with 2; occupancy stays 3 CTAs per SM, set by registers; the four-tile
// 9..10-row mode too: 8.46 ms against 8.57 with 4); the six-tile 11..16-row mode (2 CTAs per SM)
// again prefers 4 (16-row pass 9.50 -> 9.27 ms).
template <int NT>
__host__ __device__ constexpr int ring_stages() { return (NT == 0 || NT == 6) ? 4 : 2; }
constexpr int kBlockU4 = kKTileBytes / 16;    // 288 uint4 per block

// y[m][crg*256 + j] = sum over slots s = 0..ns-1, in slot order, of part[crg][s][m][j]. One
// CTA of 128 threads over M x 64 float4 columns; every load of a batch (8 slots of one
// column when M <= 2, else 4 slots of 4 columns) is issued before any is added.
__device__ __forceinline__ void vgemm_sum_slots(const VgemmParams& p, int crg, int ns) {
    const float4* src = reinterpret_cast<const float4*>(p.out.part) + (size_t)crg * p.out.max_slots * kMaxM * 64;
    const int items = p.M * 64;
    auto store = [&](int it, const float4& v) {
        const int n = crg * kCtaRows + (it & 63) * 4;
        float* o = p.y + (size_t)(it >> 6) * p.ldy + n;
        if (n < p.N) o[0] = v.x;
        if (n + 1 < p.N) o[1] = v.y;
        if (n + 2 < p.N) o[2] = v.z;
        if (n + 3 < p.N) o[3] = v.w;
    };
    auto add = [](float4& a, const float4& b) {
        a.x += b.x;
        a.y += b.y;
        a.z += b.z;
        a.w += b.w;
    };
    if (items <= kThreads) {
        const int it = threadIdx.x;
        if (it >= items) return;
        float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int s0 = 0; s0 < ns; s0 += 8) {
            float4 v[8];
#pragma unroll
            for (int k = 0; k < 8; ++k)
                if (s0 + k < ns) v[k] = __ldcg(src + ((size_t)(s0 + k) * kMaxM + (it >> 6)) * 64 + (it & 63));
#pragma unroll
            for (int k = 0; k < 8; ++k)
                if (s0 + k < ns) add(sum, v[k]);
        }
        store(it, sum);
        return;
    }
    for (int base = 0; base < items; base += 4 * kThreads) {
        float4 sum[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) sum[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int s0 = 0; s0 < ns; s0 += 4) {
            float4 v[4][4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int it = base + j * kThreads + threadIdx.x;
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    if (it < items && s0 + k < ns)
                        v[j][k] = __ldcg(src + ((size_t)(s0 + k) * kMaxM + (it >> 6)) * 64 + (it & 63));
            }
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    if (base + j * kThreads + (int)threadIdx.x < items && s0 + k < ns) add(sum[j], v[j][k]);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int it = base + j * kThreads + threadIdx.x;
            if (it < items) store(it, sum[j]);
        }
    }
}

// Per-k-tile sizes of the staged activation operands: fp16 fragments (NT = 0) or integer
// digits (NT n-tiles), and the k-tiles one 8 KB staging chunk holds.
template <int NB, int NACC, int NT>
struct BStage {
    static constexpr int frag_u4_kt = NT ? 64 * NT : 4 * NB * 32;      // uint4 per k-tile
    static constexpr int gsum_f4_kt = NT ? kMaxM : 2 * NACC * 4;       // float4 per k-tile
    static constexpr int kt = 512 / frag_u4_kt > 0 ? 512 / frag_u4_kt : 1;
    static constexpr int frag_u4 = kt * frag_u4_kt;
    static constexpr int gsum_f4 = kt * gsum_f4_kt;
};

template <int NB, int NACC, bool PACKED, int NT>
__global__ void __launch_bounds__(kThreads, (NACC == 2 || NT == 6) ? 2 : 3) vgemm_kernel(VgemmParams p) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    using BS = BStage<NB, NACC, NT>;
    constexpr int kStages = ring_stages<NT>();
    constexpr int kFragU4 = BS::frag_u4;
    constexpr int kGsumF4 = BS::gsum_f4;
    constexpr int kBufU4 = kFragU4 + kGsumF4;
    uint4* ring = reinterpret_cast<uint4*>(smem_raw);                 // [warp][stage][288]
    uint4* bbuf = ring + kWarps * kStages * kBlockU4;                 // [2][kBufU4]
    uint64_t* wbar = reinterpret_cast<uint64_t*>(bbuf + 2 * kBufU4);  // [warp][stage]
    uint64_t* bbar = wbar + kWarps * kStages;                         // [2]
    // Row groups this CTA must finish (it arrived last on them): bit i = first row group of
    // the CTA's range + i. The sums run after the streaming loop, when the accumulators are
    // dead, so their loads can all be in flight at once.
    __shared__ unsigned s_lastmask;

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int ktiles = p.out.ktiles;
    const int T = p.out.n_crg * ktiles;
    const int G = gridDim.x;
    const int c = blockIdx.x;
    const int u_begin = (int)((long long)c * T / G), u_end = (int)((long long)(c + 1) * T / G);
    const int n_units = u_end - u_begin;
    const uint4* wbase = reinterpret_cast<const uint4*>(p.w);

    if (lane == 0)
        for (int s = 0; s < kStages; ++s) mbar_init(&wbar[warp * kStages + s], 1);
    if (threadIdx.x == 0) {
        mbar_init(&bbar[0], 1);
        mbar_init(&bbar[1], 1);
    }
    if (threadIdx.x == 0) s_lastmask = 0;
    mbar_init_fence();
    __syncthreads();

    // Unit cursors advance incrementally: no integer division inside the streaming loop.
    struct Cursor {
        int u, crg, kt;
    };
    auto advance = [&](Cursor& q) {
        ++q.u;
        if (++q.kt == ktiles) { q.kt = 0; ++q.crg; }
    };
    auto active = [&](const Cursor& q) { return q.crg * kWarps + warp < p.n_wrg; };
    auto issue_w = [&](const Cursor& q, int i) {  // lane 0: unit q (the CTA's i-th) into stage i % kStages
        uint64_t* bar = &wbar[warp * kStages + (i % kStages)];
        mbar_expect_tx(bar, kKTileBytes);
        bulk_g2s(ring + (warp * kStages + (i % kStages)) * kBlockU4,
                 wbase + ((size_t)q.u * kWarps + warp) * kBlockU4, kKTileBytes, bar);
    };
    struct ChunkRec {
        int s, kt, len;
    };
    auto make_chunk = [&](int s0, int kt0) {
        ChunkRec r;
        r.s = s0;
        r.kt = kt0;
        r.len = min(min(BS::kt, ktiles - kt0), u_end - s0);
        return r;
    };
    auto next_chunk = [&](const ChunkRec& r) {
        const int kt = r.kt + r.len == ktiles ? 0 : r.kt + r.len;
        return make_chunk(r.s + r.len, kt);
    };
    auto issue_b = [&](const ChunkRec& r, int buf) {  // thread 0: activation fragments of a chunk
        const uint32_t fb = (uint32_t)r.len * BS::frag_u4_kt * 16, gb = (uint32_t)r.len * BS::gsum_f4_kt * 16;
        mbar_expect_tx(&bbar[buf], fb + gb);
        bulk_g2s(bbuf + buf * kBufU4, p.bfrag + (size_t)r.kt * BS::frag_u4_kt, fb, &bbar[buf]);
        bulk_g2s(bbuf + buf * kBufU4 + kFragU4, reinterpret_cast<const float4*>(p.gsum) + (size_t)r.kt * BS::gsum_f4_kt,
                 gb, &bbar[buf]);
    };

    Cursor cur{u_begin, u_begin / ktiles, u_begin % ktiles};
    Cursor pre = cur;  // the unit kStages ahead of `cur`
    // Let the next kernel launch now; its CTAs run only their own prologue until they wait.
    pdl_launch_dependents();
    // Weight prefetch does not depend on the previous kernel: issue it before the wait.
    for (int i = 0; i < kStages; ++i) {
        if (i < n_units && lane == 0 && active(pre)) issue_w(pre, i);
        advance(pre);
    }
    pdl_wait();

    ChunkRec chk = make_chunk(cur.u, cur.kt);
    ChunkRec nxt = next_chunk(chk);
    int ch = 0;
    if (threadIdx.x == 0 && n_units > 0) {
        issue_b(chk, 0);
        if (nxt.s < u_end) issue_b(nxt, 1);
    }
    bool failed = n_units > 0 && !mbar_wait(&bbar[0], 0);
    uint32_t wphase = 0;  // bit s: parity of the next completion of stage s

    constexpr int kJ = DigitRows<NT ? NT : 2>::J;
    float acc[kTilesPerWarp][NT ? 1 : NACC][4];          // fp16 modes
    float accd[kTilesPerWarp][NT ? kJ : 1][2];           // digit modes
#pragma unroll
    for (int r = 0; r < kTilesPerWarp; ++r) {
#pragma unroll
        for (int a = 0; a < (NT ? 1 : NACC); ++a)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[r][a][i] = 0.f;
#pragma unroll
        for (int j = 0; j < (NT ? kJ : 1); ++j) accd[r][j][0] = accd[r][j][1] = 0.f;
    }
    int seg_crg = cur.crg;
    const int g = lane >> 2, t = lane & 3;

    const int first_crg = cur.crg;
    auto flush_segment = [&](int crg) {
        const int lo = vgemm_cta_of_unit32(crg * ktiles, T, G);
        const int hi = vgemm_cta_of_unit32((crg + 1) * ktiles - 1, T, G);
        const bool direct = p.y != nullptr && lo == hi;  // this CTA owns the whole row group
        const bool act = crg * kWarps + warp < p.n_wrg;
        float* dst = direct ? p.y + (size_t)crg * kCtaRows
                            : p.out.part + ((size_t)crg * p.out.max_slots + (c - lo)) * kMaxM * kCtaRows;
        const int ld = direct ? p.ldy : kCtaRows;
        const int nmax = direct ? p.N - crg * kCtaRows : kCtaRows;
        if constexpr (NT > 0) {
            // Thread t holds activation rows t, 4+t (8+t, 12+t); with two tiles its second
            // row is row 4, with four tiles its third and fourth are rows 8 and 9, valid on
            // thread 0 only. No 2^24 factor: digits are integers.
#pragma unroll
            for (int r = 0; r < kTilesPerWarp; ++r)
#pragma unroll
                for (int j = 0; j < kJ; ++j)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int m = (NT == 2 && j == 1) ? 4 : (NT == 4 && j >= 2) ? 6 + j : 4 * j + t;
                        const bool mine = (NT != 2 || j == 0 || t == 0) && (NT != 4 || j < 2 || t == 0);
                        const int nl = warp * kWarpRows + r * 16 + g + 8 * h;
                        if (act && !failed && mine && m < p.M && nl < nmax) dst[(size_t)m * ld + nl] = accd[r][j][h];
                        accd[r][j][h] = 0.f;
                    }
        }
#pragma unroll
        for (int r = 0; r < kTilesPerWarp; ++r) {
#pragma unroll
            for (int a = 0; a < (NT ? 0 : NACC); ++a) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    float v = acc[r][a][i];
                    if (PACKED) v += __shfl_xor_sync(0xffffffffu, v, 2);
                    v *= 16777216.0f;  // 2^24: the subnormal operand scale
                    const int m = a * 8 + 2 * t + (i & 1);
                    const int nl = warp * kWarpRows + r * 16 + g + ((i >> 1) << 3);
                    if (act && !failed && (!PACKED || t < 2) && m < p.M && nl < nmax) dst[(size_t)m * ld + nl] = v;
                    acc[r][a][i] = 0.f;
                }
            }
        }
        if (p.y && !direct) {
            // Publish this slot and count the arrival; the last arrival owns the sum.
            __threadfence();
            __syncthreads();
            if (threadIdx.x == 0 && atomicAdd(p.cnt + crg, 1u) == (unsigned)(hi - lo))
                s_lastmask |= 1u << (crg - first_crg);
        }
    };

    for (int i = 0; i < n_units; ++i) {
        if (cur.u == chk.s + chk.len) {
            // Next chunk: everyone is done with chunk ch, so its buffer's successor may load.
            __syncthreads();
            ++ch;
            chk = nxt;
            nxt = next_chunk(chk);
            if (threadIdx.x == 0 && nxt.s < u_end && !failed) {
                fence_proxy_async();  // generic reads of that buffer precede the bulk write
                issue_b(nxt, (ch + 1) & 1);
            }
            if (!failed && !mbar_wait(&bbar[ch & 1], (ch >> 1) & 1)) failed = true;
        }
        if (cur.crg != seg_crg) {
            flush_segment(seg_crg);
            seg_crg = cur.crg;
        }
        const int stage = i % kStages;
        if (active(cur)) {
            uint64_t* bar = &wbar[warp * kStages + stage];
            if (!failed && !mbar_wait(bar, (wphase >> stage) & 1)) failed = true;
            wphase ^= 1u << stage;
            if (!failed) {
                const int off = cur.u - chk.s;
                const uint4* bsm = bbuf + (ch & 1) * kBufU4 + off * BS::frag_u4_kt;
                const float4* gsm = reinterpret_cast<const float4*>(bbuf + (ch & 1) * kBufU4 + kFragU4) +
                                    off * BS::gsum_f4_kt;
                if constexpr (NT > 0)
                    compute_ktile_digits<NT>(ring + (warp * kStages + stage) * kBlockU4,
                                             reinterpret_cast<const uint2*>(bsm), reinterpret_cast<const float2*>(gsm),
                                             accd, lane);
                else
                    compute_ktile<NB, NACC, PACKED>(ring + (warp * kStages + stage) * kBlockU4, bsm, gsm, acc, lane);
            }
        }
        __syncwarp();
        if (lane == 0 && !failed && i + kStages < n_units && active(pre)) {
            fence_proxy_async();
            issue_w(pre, i + kStages);
        }
        advance(cur);
        advance(pre);
    }
    if (n_units > 0) flush_segment(seg_crg);
    if (p.y) {
        __syncthreads();
        unsigned mask = s_lastmask;
        if (mask) __threadfence();
        while (mask) {
            const int crg = first_crg + __ffs(mask) - 1;
            mask &= mask - 1;
            const int lo = vgemm_cta_of_unit32(crg * ktiles, T, G);
            const int hi = vgemm_cta_of_unit32((crg + 1) * ktiles - 1, T, G);
            vgemm_sum_slots(p, crg, hi - lo + 1);
            if (threadIdx.x == 0) p.cnt[crg] = 0;  // every CTA of the group has arrived
        }
    }
    if (failed && p.err) atomicExch(p.err, 1);
}

template <int NB, int NACC, int NT>
static constexpr size_t smem_bytes() {
    using BS = BStage<NB, NACC, NT>;
    constexpr int kStages = ring_stages<NT>();
    return (size_t)kWarps * kStages * kKTileBytes + 2 * ((size_t)BS::frag_u4 * 16 + (size_t)BS::gsum_f4 * 16) +
           (kWarps * kStages + 2) * sizeof(uint64_t);
}

template <int NB, int NACC, bool PACKED, int NT>
static int max_ctas_per_sm() {
    static int cached = -1;
    if (cached < 0) {
        const size_t sm = smem_bytes<NB, NACC, NT>();
        cudaFuncSetAttribute(vgemm_kernel<NB, NACC, PACKED, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        int n = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, vgemm_kernel<NB, NACC, PACKED, NT>, kThreads, sm);
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

template <int NB, int NACC, bool PACKED, int NT>
static cudaError_t launch_t(const VgemmParams& p, cudaStream_t st, bool pdl) {
    max_ctas_per_sm<NB, NACC, PACKED, NT>();  // sets the dynamic shared memory attribute once
    return launch(vgemm_kernel<NB, NACC, PACKED, NT>, dim3(p.out.grid), dim3(kThreads), smem_bytes<NB, NACC, NT>(), st,
                  pdl, p);
}

}  // namespace g4b

using namespace g4b;

int vgemm_grid(int M, int n_crg, int ktiles) {
    const BMode md = bmode_for(M);
    int per_sm;
    if (md.packed) per_sm = max_ctas_per_sm<1, 1, true, 0>();
    else if (md.nt == 2) per_sm = max_ctas_per_sm<0, 0, false, 2>();
    else if (md.nt == 3) per_sm = max_ctas_per_sm<0, 0, false, 3>();
    else if (md.nt == 4) per_sm = max_ctas_per_sm<0, 0, false, 4>();
    else per_sm = max_ctas_per_sm<0, 0, false, 6>();
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

int vgemm_plan_slots(int n_crg, int ktiles) {
    int s = 0;
    for (int M : {1, 5, 16}) s = std::max(s, vgemm_max_slots(vgemm_grid(M, n_crg, ktiles), n_crg, ktiles));
    return s;
}

cudaError_t vgemm_launch(const VgemmParams& p, cudaStream_t st, bool pdl) {
    if (p.M < 1 || p.M > kMaxM) return cudaErrorInvalidValue;
    if (p.y && (!p.cnt || p.ldy < p.N)) return cudaErrorInvalidValue;
    // A CTA records the row groups it must finish in a 32-bit mask: its unit range may touch
    // at most 32 of them (n_crg / grid + 2 bounds the count).
    if (p.y && p.out.n_crg / p.out.grid + 2 > 32) return cudaErrorInvalidValue;
    // The kernel's 32-bit unit-to-CTA arithmetic needs (T + 1) * G < 2^31.
    if (((long long)p.out.n_crg * p.out.ktiles + 1) * p.out.grid >= (1ll << 31)) return cudaErrorInvalidValue;
    if (vgemm_max_slots(p.out.grid, p.out.n_crg, p.out.ktiles) > p.out.max_slots) return cudaErrorInvalidValue;
    const BMode md = bmode_for(p.M);
    if (md.packed) return launch_t<1, 1, true, 0>(p, st, pdl);
    if (md.nt == 2) return launch_t<0, 0, false, 2>(p, st, pdl);
    if (md.nt == 3) return launch_t<0, 0, false, 3>(p, st, pdl);
    if (md.nt == 4) return launch_t<0, 0, false, 4>(p, st, pdl);
    return launch_t<0, 0, false, 6>(p, st, pdl);
}
