// Long-context attention for the full-attention layers (head_dim 512, bf16 KV cache) on the
// 5th-generation tensor cores: Attention.hlsl (shaders/Attention.hlsl:65-179) for verify
// batches of up to 16 rows at tens of thousands of cached keys, where the KV read dominates.
//
// Grid: one CTA per (key split, row group, KV head). A row group is gqa / G query heads of the
// KV head over the batch's positions (verify batches, up to 48 rows: row r = m * heads + j) or,
// for a prefill chunk, one query head over a block of up to 48 consecutive positions. S splits
// share the group's key range [0, base + its last position] in 128-key tiles, and every K/V tile
// a CTA loads serves all of its rows.
// Per tile, with warp roles:
//   * warp 0 (one thread) streams the tile's K, then the previous tile's V, through a ring of
//     three 32 KB slots: each slot is two TMA tensor copies of 128 keys x 64 dims in the
//     128-byte-swizzled layout (no multicast);
//   * warp 1 (one thread) issues the MMAs: S^T[key][row] = K Q^T into one of two TMEM buffers,
//     with the fp32 query split into two bf16 terms (q = q1 + q2, 16 significant bits), then
//     O^T[dim][row] += V^T P^T into four TMEM tiles of 128 dims (V read MN-major, P as two bf16
//     terms);
//   * warps 4..11 (TMEM lanes = keys, columns = rows; two warps per lane quadrant, 24 rows each)
//     read S^T, keep the online softmax (running max and sum in fp32, exp of the fp32 scores;
//     the per-row reductions over a warp's 32 keys are butterfly reduce-scatters), write P^T to
//     shared memory and, when a row's maximum rises by more than kLcLazy, rescale that row of
//     O^T in TMEM before the tile's P V is issued;
//   * warps 2..11 stage the query terms first.
// Each CTA writes its unnormalised O and {max, sum} per row; a second kernel combines the splits
// (the softmax-weighted sum) and writes the o-projection's B fragments (the wide layout for a
// prefill chunk).
//
// Row m of the batch sits at position base + m and sees keys [0, base + m]. Every wait is bounded
// (2 s); a CTA that gives up records kErrAttnLc in the error word and leaves.
#include <cuda.h>
#include <cuda_bf16.h>

#include "bfrag.cuh"
#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"
#include "model_dev.h"
#include "tcgen05.cuh"
#include "tma.cuh"

#include <algorithm>
#include <cstdlib>
#include <cstring>

namespace g4b {

namespace {

constexpr int kLcHd = 512;
constexpr int kLcKeys = 128;    // keys per tile: the M of S^T
constexpr int kLcMaxN = 48;     // query rows per CTA
constexpr int kLcSlots = 3;
constexpr uint32_t kLcBoxBytes = kLcKeys * 128;      // 128 keys x 64 dims of bf16
constexpr uint32_t kLcSlotBytes = 2 * kLcBoxBytes;   // 128 dims
constexpr uint32_t kLcRingBytes = kLcSlots * kLcSlotBytes;
constexpr uint32_t kLcQBytes = 2 * (kLcHd / 64) * kLcMaxN * 128;  // 2 terms x 8 dim blocks x N rows
constexpr uint32_t kLcPBytes = 2 * 2 * kLcMaxN * 128;             // 2 terms x 2 key blocks x N rows
constexpr int kLcThreads = 384;
constexpr int kLcSoftWarps = 8;   // warps 4..11
constexpr int kLcStageWarps = 10;  // warps 2..11
constexpr uint32_t kLcTmemCols = 512;
constexpr int kErrAttnLc = 7;
constexpr float kLcLazy = 8.0f;  // rescale threshold of the running maximum (natural-log units)

struct LcCtl {
    uint64_t full[kLcSlots], empty[kLcSlots];
    uint64_t s_full[2], s_free[2];
    uint64_t q_ready, p_full, o_done, done;
    uint32_t tmem_base;
    int abort;
    int changed;
    float m_run[kLcMaxN], l_run[kLcMaxN], m_new[kLcMaxN], corr[kLcMaxN];
    float red[4][kLcMaxN];
};
constexpr size_t kLcSmemBytes = 1024 + kLcRingBytes + kLcQBytes + kLcPBytes + sizeof(LcCtl);
static_assert(kLcSmemBytes <= 232448, "long-context attention exceeds the shared-memory limit");

// Bounded wait that also gives up as soon as another warp of the CTA has.
__device__ __forceinline__ bool lc_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    while (!mbar_try_wait_sleep(bar, parity, 1000000u)) {
        if (*abort) return false;
        if (global_ns() - t0 > kWaitLimitNs) {
            *abort = 1;
            if (err) atomicExch(err, kErrAttnLc);
            return false;
        }
    }
    return true;
}

// Barrier of the eight softmax warps; returns the AND of `ok` over their 256 threads.
__device__ __forceinline__ bool sm_bar_and(bool ok) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.b32 p, %1, 0;\n bar.red.and.pred q, 1, 256, p;\n selp.u32 %0, 1, 0, q;\n}"
        : "=r"(r)
        : "r"((uint32_t)ok)
        : "memory");
    return r != 0;
}
__device__ __forceinline__ void sm_bar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// Reduce-scatter of 24 per-lane values over the warp (max or sum across the 32 lanes): each
// exchange sends the half the lane gives away and combines the half it keeps, so 27 shuffles
// replace 24 x 5. Afterwards v[0..2] hold the reductions of rows 12 b4 + 6 b3 + 3 b2 + (0..2),
// b_i the lane's bits (the four lanes sharing bits 4..2 hold the same values).
template <bool kMax>
__device__ __forceinline__ void reduce_scatter24(float (&v)[24], int lane) {
    auto op = [](float a, float b) { return kMax ? fmaxf(a, b) : a + b; };
    {
        const bool h = lane & 16;
#pragma unroll
        for (int i = 0; i < 12; ++i) {
            const float snd = h ? v[i] : v[i + 12], kp = h ? v[i + 12] : v[i];
            v[i] = op(kp, __shfl_xor_sync(0xffffffffu, snd, 16));
        }
    }
    {
        const bool h = lane & 8;
#pragma unroll
        for (int i = 0; i < 6; ++i) {
            const float snd = h ? v[i] : v[i + 6], kp = h ? v[i + 6] : v[i];
            v[i] = op(kp, __shfl_xor_sync(0xffffffffu, snd, 8));
        }
    }
    {
        const bool h = lane & 4;
#pragma unroll
        for (int i = 0; i < 3; ++i) {
            const float snd = h ? v[i] : v[i + 3], kp = h ? v[i + 3] : v[i];
            v[i] = op(kp, __shfl_xor_sync(0xffffffffu, snd, 4));
        }
    }
#pragma unroll
    for (int i = 0; i < 3; ++i) {
        v[i] = op(v[i], __shfl_xor_sync(0xffffffffu, v[i], 2));
        v[i] = op(v[i], __shfl_xor_sync(0xffffffffu, v[i], 1));
    }
}

// One 3-D TMA tensor copy (x = dim, y = KV head, z = position) completing on `bar`.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ uint16_t bf16_bits(float x) { return __bfloat16_as_ushort(__float2bfloat16_rn(x)); }
__device__ __forceinline__ float bf16_val(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

// Byte offset of element (row, col) of a [rows][64] bf16 block in the 128-byte-swizzled layout.
__device__ __forceinline__ uint32_t sw128_off(int row, int col) {
    return (uint32_t)row * 128 + ((uint32_t)(((col >> 3) ^ (row & 7))) << 4) + (uint32_t)(col & 7) * 2;
}

__global__ void __launch_bounds__(kLcThreads, 1)
    attn_lc_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                   AttnLcParams p) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    unsigned char* ring = sm;
    unsigned char* qs = ring + kLcRingBytes;
    unsigned char* pt = qs + kLcQBytes;
    LcCtl& c = *reinterpret_cast<LcCtl*>(pt + kLcPBytes);
    volatile int* abort = &c.abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int split = blockIdx.x, grp = blockIdx.y / p.BM, kvh_i = blockIdx.z;
    const int m0 = (blockIdx.y % p.BM) * p.mb, mcnt = min(p.M - m0, p.mb);  // this group's positions
    const int N = p.N, hpg = p.hpg, R = mcnt * hpg;
    const int gqa = p.qh / p.kvh;
    // base_pos stays fixed during a pass (only a pass's last kernel writes it), so it is read
    // before waiting on the producer of the query rows.
    const int base = p.sp->base_pos;
    const int kmax = base + m0 + mcnt;  // the group's last row sees keys up to base + m0 + mcnt - 1
    const int per = ((kmax + p.S - 1) / p.S + kLcKeys - 1) / kLcKeys * kLcKeys;
    const int ks = split * per, ke = min(kmax, ks + per);
    const int T = ks < ke ? (ke - ks + kLcKeys - 1) / kLcKeys : 0;
    const int cta = (kvh_i * p.G * p.BM + (int)blockIdx.y) * p.S + split;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kLcSlots; ++s) {
            mbar_init(&c.full[s], 1);
            mbar_init(&c.empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&c.s_full[b], 1);
            mbar_init(&c.s_free[b], kLcSoftWarps);
        }
        mbar_init(&c.q_ready, kLcStageWarps);
        mbar_init(&c.p_full, kLcSoftWarps);
        mbar_init(&c.o_done, 1);
        mbar_init(&c.done, 1);
        c.abort = 0;
        c.changed = 0;
        for (int r = 0; r < kLcMaxN; ++r) {
            c.m_run[r] = -INFINITY;
            c.l_run[r] = 0.f;
        }
        mbar_init_fence();
    }
    if (warp == 1) tc::alloc(&c.tmem_base, kLcTmemCols);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = c.tmem_base;
    const uint32_t s_col = 0, o_col = 2 * (uint32_t)N;  // S^T buffers, then the four O^T tiles
    pdl_launch_dependents();

    if (warp == 0) {
        // ------------------------------------------------------------------ producer
        if (lane == 0) {
            int q = 0;
            bool ok = true, waited = false;
            auto load = [&](const CUtensorMap* map, int kt, int ci) {
                const int slot = q % kLcSlots;
                if (q >= kLcSlots && !lc_wait(&c.empty[slot], ((q / kLcSlots) + 1) & 1, abort, p.err)) return false;
                unsigned char* dst = ring + slot * kLcSlotBytes;
                mbar_expect_tx(&c.full[slot], kLcSlotBytes);
                tma_load_3d(dst, map, 128 * ci, kvh_i, kt, &c.full[slot]);
                tma_load_3d(dst + kLcBoxBytes, map, 128 * ci + 64, kvh_i, kt, &c.full[slot]);
                ++q;
                return true;
            };
            // Order of use: K(0), then for each t >= 1 K(t) and V(t - 1), then V(T - 1). Keys
            // below base come from earlier passes and are fetched before the producer wait.
            for (int t = 0; t <= T && ok; ++t) {
                if (t < T) {
                    const int kt = ks + t * kLcKeys;
                    if (!waited && kt + kLcKeys > base) {
                        pdl_wait();
                        waited = true;
                    }
                    for (int ci = 0; ci < 4 && ok; ++ci) ok = load(&kmap, kt, ci);
                }
                if (t >= 1)
                    for (int ci = 0; ci < 4 && ok; ++ci) ok = load(&vmap, ks + (t - 1) * kLcKeys, ci);
            }
            // Every issued copy lands before the CTA can exit.
            for (int i = max(0, q - kLcSlots); i < q; ++i)
                if (!mbar_wait(&c.full[i % kLcSlots], (i / kLcSlots) & 1) && p.err) atomicExch(p.err, kErrAttnLc);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t id_s = tc::idesc_bf16(kLcKeys, N, false), id_o = tc::idesc_bf16(128, N, true);
            const uint32_t q_addr = smem_u32(qs), p_addr = smem_u32(pt), r_addr = smem_u32(ring);
            const uint32_t blk = (uint32_t)N * 128;  // bytes of one [N rows][64] block
            int q = 0;
            bool ok = lc_wait(&c.q_ready, 0, abort, p.err);
            auto issue_s = [&](int t) {
                const int b = t & 1;
                if (t >= 2 && !lc_wait(&c.s_free[b], ((t >> 1) - 1) & 1, abort, p.err)) return false;
                for (int ci = 0; ci < 4; ++ci, ++q) {
                    const int slot = q % kLcSlots;
                    if (!lc_wait(&c.full[slot], (q / kLcSlots) & 1, abort, p.err)) return false;
                    tc::fence_after_sync();
                    const uint32_t sa = r_addr + slot * kLcSlotBytes;
#pragma unroll
                    for (int h = 0; h < 2; ++h)
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
#pragma unroll
                            for (int term = 0; term < 2; ++term) {
                                const uint32_t qb = q_addr + (uint32_t)(term * 8 + 2 * ci + h) * blk + kk * 32;
                                tc::mma_ss(tmem + s_col + b * N, tc::desc_sw128(sa + h * kLcBoxBytes + kk * 32),
                                           tc::desc_sw128(qb), id_s, (ci | h | kk | term) ? 1u : 0u);
                            }
                    tc::commit(&c.empty[slot]);
                }
                tc::commit(&c.s_full[b]);
                return true;
            };
            auto issue_o = [&](int t) {
                if (!lc_wait(&c.p_full, t & 1, abort, p.err)) return false;
                tc::fence_after_sync();
                for (int ci = 0; ci < 4; ++ci, ++q) {
                    const int slot = q % kLcSlots;
                    if (!lc_wait(&c.full[slot], (q / kLcSlots) & 1, abort, p.err)) return false;
                    tc::fence_after_sync();
                    const uint32_t sa = r_addr + slot * kLcSlotBytes;
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk)
#pragma unroll
                        for (int term = 0; term < 2; ++term) {
                            // V^T rows = this slot's 128 dims (two 64-dim boxes kLcBoxBytes apart),
                            // K = keys 16 kk .. 16 kk + 15 (rows of the boxes, 8-key groups 1 KB apart).
                            const uint64_t a = tc::desc_sw128_mn(sa + kk * 2048, kLcBoxBytes, 1024);
                            const uint32_t pb = p_addr + (uint32_t)(term * 2 + (kk >> 2)) * blk + (kk & 3) * 32;
                            tc::mma_ss(tmem + o_col + ci * N, a, tc::desc_sw128(pb), id_o,
                                       (t > 0 || kk > 0 || term > 0) ? 1u : 0u);
                        }
                    tc::commit(&c.empty[slot]);
                }
                tc::commit(&c.o_done);
                return true;
            };
            if (ok && T > 0) ok = issue_s(0);
            for (int t = 1; t < T && ok; ++t) ok = issue_s(t) && issue_o(t - 1);
            if (ok && T > 0) ok = issue_o(T - 1);
            tc::commit(&c.done);  // every MMA has completed before tensor memory is freed
            if (!mbar_wait(&c.done, 0) && p.err) atomicExch(p.err, kErrAttnLc);
        }
    } else {
        // ------------------------------------------------------------------ query staging
        pdl_wait();
        for (int r = warp - 2; r < N; r += kLcStageWarps) {
            float x[16];
            if (r < R) {
                const int m = m0 + r / hpg, qhead = kvh_i * gqa + grp * hpg + r % hpg;
                const float4* src = reinterpret_cast<const float4*>(p.q + ((size_t)m * p.qh + qhead) * kLcHd) + 4 * lane;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float4 v = src[i];
                    x[4 * i] = v.x;
                    x[4 * i + 1] = v.y;
                    x[4 * i + 2] = v.z;
                    x[4 * i + 3] = v.w;
                }
            } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) x[i] = 0.f;
            }
            // dims 16 lane .. 16 lane + 15: chunks 2 lane, 2 lane + 1 of dim block lane / 4
            const int db = lane >> 2;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                uint32_t hi[4], lo[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    uint16_t a0 = bf16_bits(x[8 * h + 2 * i]), a1 = bf16_bits(x[8 * h + 2 * i + 1]);
                    uint16_t b0 = bf16_bits(x[8 * h + 2 * i] - bf16_val(a0));
                    uint16_t b1 = bf16_bits(x[8 * h + 2 * i + 1] - bf16_val(a1));
                    hi[i] = (uint32_t)a0 | ((uint32_t)a1 << 16);
                    lo[i] = (uint32_t)b0 | ((uint32_t)b1 << 16);
                }
                const int col = (lane & 3) * 16 + 8 * h;
                const uint32_t off = sw128_off(r, col);
                *reinterpret_cast<uint4*>(qs + (size_t)(0 * 8 + db) * N * 128 + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                *reinterpret_cast<uint4*>(qs + (size_t)(1 * 8 + db) * N * 128 + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            }
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(&c.q_ready);

        if (warp >= 4) {
            // -------------------------------------------------------------- softmax
            const int sw = warp - 4, qd = warp & 3, half = sw >> 2;
            const int tid = sw * 32 + lane;  // 0..255
            const int r0 = 24 * half;        // this warp's rows r0 .. r0 + 23
            const bool active = r0 < N;      // warp-uniform
            const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
            const int rs0 = r0 + ((lane >> 4) & 1) * 12 + ((lane >> 3) & 1) * 6 + ((lane >> 2) & 1) * 3;
            const int kb = (qd * 32 + lane) >> 6, col = (qd * 32 + lane) & 63;
            float s[24];
            bool ok = true;
            for (int t = 0; t < T; ++t) {
                const int b = t & 1;
                const int kt = ks + t * kLcKeys, key = kt + qd * 32 + lane;
                ok = sm_bar_and(ok && lc_wait(&c.s_full[b], (t >> 1) & 1, abort, p.err));
                if (!ok) break;
                tc::fence_after_sync();
                if (active) {
                    float v[16], w[8];
                    tc::ld16(tmem + lane_base + s_col + b * N + r0, v);
                    tc::ld8(tmem + lane_base + s_col + b * N + r0 + 16, w);
                    tc::wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j) s[j] = v[j];
#pragma unroll
                    for (int j = 0; j < 8; ++j) s[16 + j] = w[j];
                }
                tc::fence_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive(&c.s_free[b]);
                // Masked, scaled scores. A tile below every row's last key and inside the split
                // needs the row check only.
                const bool inside = kt + kLcKeys <= ke && kt + kLcKeys - 1 <= base + m0;
                float red[24];
#pragma unroll
                for (int j = 0; j < 24; ++j) {
                    const int r = r0 + j;
                    const bool valid = r < R && (inside || (key < ke && key <= base + m0 + r / hpg));
                    s[j] = valid ? s[j] * p.scale : -INFINITY;
                    red[j] = s[j];
                }
                reduce_scatter24<true>(red, lane);
                if (active && (lane & 3) == 0)
#pragma unroll
                    for (int i = 0; i < 3; ++i) c.red[qd][rs0 + i] = red[i];
                sm_bar();
                if (tid < N) {
                    // The row's reference maximum moves only when a score exceeds it by more than
                    // kLcLazy (so p <= e^kLcLazy); O^T and the sum are kept relative to it, which
                    // leaves their ratio exact and skips most rescales.
                    const float mt = fmaxf(fmaxf(c.red[0][tid], c.red[1][tid]), fmaxf(c.red[2][tid], c.red[3][tid]));
                    const float mo = c.m_run[tid];
                    const float mn = (mo == -INFINITY || mt > mo + kLcLazy) ? fmaxf(mo, mt) : mo;
                    c.m_new[tid] = mn;
                    c.corr[tid] = mn == mo ? 1.f : expf(mo - mn);  // 0 while nothing was seen
                    if (t > 0 && mn != mo) c.changed = 1;
                }
                sm_bar();
                const bool rescale = c.changed != 0;
                // P and its row sums need only this tile's scores: they are computed while the
                // previous tile's P V may still run. Only the stores into the single P^T buffer
                // and the O^T rescale wait for it.
#pragma unroll
                for (int j = 0; j < 24; ++j) {
                    const int r = r0 + j;
                    float pr = 0.f;
                    if (active && r < N && s[j] != -INFINITY) pr = expf(s[j] - c.m_new[r]);
                    const uint16_t h1 = bf16_bits(pr), h2 = bf16_bits(pr - bf16_val(h1));
                    s[j] = pr;
                    red[j] = bf16_val(h1) + bf16_val(h2);
                }
                reduce_scatter24<false>(red, lane);
                if (active && (lane & 3) == 0)
#pragma unroll
                    for (int i = 0; i < 3; ++i) c.red[qd][rs0 + i] = red[i];
                ok = sm_bar_and(ok && (t == 0 || lc_wait(&c.o_done, (t - 1) & 1, abort, p.err)));
                if (!ok) break;
                tc::fence_after_sync();
                if (active) {
#pragma unroll
                    for (int j = 0; j < 24; ++j) {
                        const int r = r0 + j;
                        if (r >= N) break;
                        const uint16_t h1 = bf16_bits(s[j]), h2 = bf16_bits(s[j] - bf16_val(h1));
                        const uint32_t off = sw128_off(r, col);
                        *reinterpret_cast<uint16_t*>(pt + (size_t)(0 * 2 + kb) * N * 128 + off) = h1;
                        *reinterpret_cast<uint16_t*>(pt + (size_t)(1 * 2 + kb) * N * 128 + off) = h2;
                    }
                }
                if (rescale) {
                    // This warp's two O^T tiles (dims 128 ci .. +127, lane = dim) times corr[row].
#pragma unroll 1
                    for (int ci = half; ci < 4; ci += 2)
#pragma unroll
                        for (int i = 0; i < kLcMaxN / 16; ++i)
                            if (16 * i < N) {
                                float v[16];
                                const uint32_t ta = tmem + lane_base + o_col + ci * N + 16 * i;
                                tc::ld16(ta, v);
                                tc::wait_ld();
#pragma unroll
                                for (int j = 0; j < 16; ++j) v[j] *= c.corr[16 * i + j];
                                tc::st16(ta, v);
                            }
                    tc::wait_st();
                }
                if (tid < N) {
                    c.l_run[tid] = c.l_run[tid] * c.corr[tid] + (c.red[0][tid] + c.red[1][tid]) + (c.red[2][tid] + c.red[3][tid]);
                    c.m_run[tid] = c.m_new[tid];
                }
                if (tid == 0) c.changed = 0;  // every thread read it before the barrier above
                fence_proxy_async();
                tc::fence_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive(&c.p_full);
            }
            // This split's partial result: O^T (lane = dim) and {max, sum} per row.
            ok = sm_bar_and(ok && (T == 0 || lc_wait(&c.o_done, (T - 1) & 1, abort, p.err)));
            if (ok && T > 0) {
                tc::fence_after_sync();
                float* dst = p.part + (size_t)cta * N * kLcHd;
#pragma unroll 1
                for (int ci = half; ci < 4; ci += 2)
#pragma unroll
                    for (int i = 0; i < kLcMaxN / 16; ++i)
                        if (16 * i < N) {
                            float v[16];
                            tc::ld16(tmem + lane_base + o_col + ci * N + 16 * i, v);
                            tc::wait_ld();
#pragma unroll
                            for (int j = 0; j < 16; ++j)
                                if (16 * i + j < R)
                                    __stcg(dst + (size_t)(16 * i + j) * kLcHd + 128 * ci + qd * 32 + lane, v[j]);
                        }
            }
            if (tid < N) p.ml[(size_t)cta * N + tid] = ok && T > 0 ? make_float2(c.m_run[tid], c.l_run[tid])
                                                                : make_float2(-INFINITY, 0.f);
        }
    }

    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::dealloc(tmem, kLcTmemCols);
    }
}

// out[row] = sum_s e^(m_s - M) O_s / sum_s e^(m_s - M) l_s, one warp per (row, 64-dim group),
// written as the o-projection's B fragments.
__global__ void __launch_bounds__(256) attn_lc_combine_kernel(AttnLcParams p, void* bfrag) {
    __shared__ __half stage[8][128];
    pdl_launch_dependents();
    pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gqa = p.qh / p.kvh, rows = p.M * gqa;
    const int w = blockIdx.x * 8 + warp;
    if (w >= p.kvh * rows * 8) return;  // warp-uniform
    const int gi = w & 7, rr = (w >> 3) % rows, kvh_i = (w >> 3) / rows;
    const int m = rr / gqa, jj = rr % gqa, grp = jj / p.hpg, mbk = m / p.mb;
    const int r = (m - mbk * p.mb) * p.hpg + jj % p.hpg;
    const int cta0 = (kvh_i * p.G * p.BM + grp * p.BM + mbk) * p.S;
    // The splits' {max, sum} are spread over the lanes (32 splits per round); each lane's weight
    // then reaches the whole warp by shuffle, so the partial-output loads are independent and
    // four stay in flight. Empty splits (sum 0) never wrote a partial output and are skipped.
    float mx = -INFINITY;
    for (int s0 = 0; s0 < p.S; s0 += 32) {
        const int s = s0 + lane;
        if (s < p.S) {
            const float2 ml = p.ml[(size_t)(cta0 + s) * p.N + r];
            if (ml.y > 0.f) mx = fmaxf(mx, ml.x);
        }
    }
    mx = warp_max(mx);
    float n0 = 0.f, n1 = 0.f, den = 0.f;
    const float* col = p.part + (size_t)r * kLcHd + gi * 64 + 2 * lane;
    for (int s0 = 0; s0 < p.S; s0 += 32) {
        const int s = s0 + lane;
        float w = 0.f, lw = 0.f;
        if (s < p.S) {
            const float2 ml = p.ml[(size_t)(cta0 + s) * p.N + r];
            if (ml.y > 0.f) {
                w = expf(ml.x - mx);
                lw = w * ml.y;
            }
        }
        den += warp_sum(lw);
        const int cnt = min(32, p.S - s0);
        for (int j = 0; j < cnt; j += 4) {
            float wj[4];
            float2 o[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                wj[u] = __shfl_sync(0xffffffffu, w, (j + u) & 31);
                o[u] = make_float2(0.f, 0.f);
                if (j + u < cnt && wj[u] != 0.f)
                    o[u] = __ldcg(reinterpret_cast<const float2*>(col + (size_t)(cta0 + s0 + j + u) * p.N * kLcHd));
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (j + u >= cnt) wj[u] = 0.f;
                n0 = fmaf(wj[u], o[u].x, n0);
                n1 = fmaf(wj[u], o[u].y, n1);
            }
        }
    }
    const float inv = den > 0.f ? 1.0f / den : 0.f;
    const int K = p.qh * kLcHd;
    const BFragView bv = bfrag_view(bfrag, (K + 127) / 128 * 128, p.M);
    const int qhead = kvh_i * gqa + jj;
    if (p.M > kMaxM) {
        // Prefill rows: one static scale per row. Every output is a convex combination of cached
        // V rows, and V is RMS-normalised without a weight, so |o| <= sqrt(head_dim) (times the
        // cache's rounding, well inside 1.01).
        const float wide_e = wide_row_scale(sqrtf((float)kLcHd) * 1.01f);
        wide_store_group(bv, m, (qhead * kLcHd) / 64 + gi, n0 * inv, n1 * inv, 1.0f / wide_e);
        if (lane == 0 && qhead == 0 && gi == 0) bv.erow[m] = wide_e;
    } else {
        bfrag_store_group(bv, p.M, m, (qhead * kLcHd) / 64 + gi, n0 * inv, n1 * inv, stage[warp]);
    }
}

int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

int splits_for(int kvh, int groups) { return std::max(1, sm_count() / std::max(1, kvh * groups)); }

// Row groups of a batch of M rows: the fewest head groups whose rows (M x heads) fit a CTA; a
// prefill chunk too long for that takes one head per group over blocks of 48 positions.
struct LcShape {
    int G, BM, mb;
};
bool lc_shape(int M, int gqa, LcShape& sh) {
    if (M < 1 || M > kPrefillRows || gqa < 1) return false;
    for (int G = 1; G <= gqa; ++G)
        if (gqa % G == 0 && M * (gqa / G) <= kLcMaxN) {
            sh = {G, 1, M};
            return true;
        }
    sh = {gqa, (M + kLcMaxN - 1) / kLcMaxN, kLcMaxN};
    return true;
}

}  // namespace

int attn_lc_groups(int M, int gqa) {
    LcShape sh;
    return lc_shape(M, gqa, sh) ? sh.G * sh.BM : 0;
}

void attn_lc_scratch(int qh, int kvh, size_t* part_bytes, size_t* ml_bytes) {
    size_t pb = 0, mb = 0;
    const int gqa = qh / kvh;
    for (int M = 1; M <= kPrefillRows; ++M) {
        LcShape sh;
        if (!lc_shape(M, gqa, sh)) continue;
        const int N = (std::min(M, sh.mb) * (gqa / sh.G) + 15) / 16 * 16;
        const size_t ctas = (size_t)kvh * sh.G * sh.BM * splits_for(kvh, sh.G * sh.BM);
        pb = std::max(pb, ctas * N * kLcHd * sizeof(float));
        mb = std::max(mb, ctas * N * sizeof(float2));
    }
    *part_bytes = pb;
    *ml_bytes = mb;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against libcuda).
cudaError_t make_kv_tmap(KvTmap* out, const uint16_t* ring, int hd, int kvh, int cap) {
    using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
    static EncodeFn encode = nullptr;
    if (!encode) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        const cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) return cudaErrorNotSupported;
        encode = reinterpret_cast<EncodeFn>(fn);
    }
    static_assert(sizeof(KvTmap) == sizeof(CUtensorMap), "KvTmap must hold a CUtensorMap");
    if (hd % 64 || reinterpret_cast<uintptr_t>(ring) % 16) return cudaErrorInvalidValue;
    const cuuint64_t dims[3] = {(cuuint64_t)hd, (cuuint64_t)kvh, (cuuint64_t)cap};
    const cuuint64_t strides[2] = {(cuuint64_t)hd * 2, (cuuint64_t)kvh * hd * 2};
    const cuuint32_t box[3] = {64, 1, (cuuint32_t)kLcKeys};
    const cuuint32_t estride[3] = {1, 1, 1};
    CUtensorMap m;
    const CUresult r = encode(&m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<uint16_t*>(ring), dims, strides, box,
                              estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
    std::memcpy(out, &m, sizeof(m));
    return cudaSuccess;
}

cudaError_t attention_lc(const AttnArgs& a, const KvTmap& k, const KvTmap& v, float* part, float2* ml, int* err,
                         void* bfrag, cudaStream_t st, bool pdl) {
    if (a.hd != kLcHd || a.window != 0 || !a.kv_bf16 || a.kvh < 1 || a.qh % a.kvh) return cudaErrorInvalidValue;
    const int gqa = a.qh / a.kvh;
    LcShape sh;
    if (!lc_shape(a.M, gqa, sh)) return cudaErrorInvalidValue;
    const int G = sh.G;
    AttnLcParams p{};
    p.q = a.q;
    p.sp = a.sp;
    p.part = part;
    p.ml = ml;
    p.err = err;
    p.M = a.M;
    p.qh = a.qh;
    p.kvh = a.kvh;
    p.G = G;
    p.BM = sh.BM;
    p.mb = sh.mb;
    p.S = splits_for(a.kvh, G * sh.BM);
    // G4DENSE_ATTN_LC_SPLITS lowers the split count (never raises it past what the scratch
    // holds), so a moderate context still gives each CTA several tiles.
    if (const char* f = std::getenv("G4DENSE_ATTN_LC_SPLITS"); f && std::atoi(f) > 0) p.S = std::min(p.S, std::atoi(f));
    p.hpg = gqa / G;
    p.N = (std::min(a.M, sh.mb) * p.hpg + 15) / 16 * 16;
    p.scale = a.scale;
    static bool attr = false;
    if (!attr) {
        const cudaError_t e =
            cudaFuncSetAttribute(attn_lc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kLcSmemBytes);
        if (e != cudaSuccess) return e;
        attr = true;
    }
    CUtensorMap km, vm;
    std::memcpy(&km, &k, sizeof(km));
    std::memcpy(&vm, &v, sizeof(vm));
    cudaError_t e =
        launch(attn_lc_kernel, dim3(p.S, G * sh.BM, a.kvh), dim3(kLcThreads), kLcSmemBytes, st, pdl, km, vm, p);
    if (e != cudaSuccess) return e;
    const int warps = a.kvh * a.M * gqa * 8;
    return launch(attn_lc_combine_kernel, dim3((warps + 7) / 8), dim3(256), 0, st, pdl, p, bfrag);
}

}  // namespace g4b
