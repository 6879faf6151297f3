// Multi-row GQA attention over the KV ring -- Attention.hlsl (shaders/Attention.hlsl:65-179)
// rebuilt so the KV cache is read ONCE per KV head for all M verify rows and all of that
// head's query heads (the reference dispatches one group per (row, query head), re-reading
// the cache M * q_heads/kv_heads times).
//
// Grid: one thread-block cluster of S CTAs per (KV head, chunk of 16 query rows); CTA r of the
// cluster takes the r-th share of the batch's key range, in 64-key tiles. S (16, 12 or 8) is
// the largest size whose clusters all fit on the GPU at once (one wave). Per tile:
//   * K and V land in shared memory by cp.async;
//   * S = Q K^T on the tensor cores (mma.sync m16n8k16, fp32 accumulate), warp w taking keys
//     8w..8w+7. The cached K is exact in the MMA's input type (FP16, or bf16 in long-context
//     mode); the fp32 query is split into 2 terms q = q1 + q2 after a power-of-two row
//     scaling, so the scores carry the query to 22 significant bits (FP16) or 16 (bf16);
//   * an online softmax per row (running max / sum in fp32, exp of the fp32 scores), warp w
//     taking rows 2w, 2w+1;
//   * O += P V on the tensor cores with P (scaled by 2^14) split the same way, warp w owning
//     columns [w*hd/8, (w+1)*hd/8) of the output.
// The cluster's partial results are then combined through distributed shared memory and
// written directly as the o-projection's B fragments.
//
// Row m of the batch sits at position base+m and sees keys [max(0, base+m+1-window),
// base+m+1) (all keys from 0 on full-attention layers): the reference's per-row causal span
// (shaders/Attention.hlsl:82-86). Scale is a parameter (1.0 for Gemma 4,
// src/cpu_reference.cpp:508-510).
#include <cooperative_groups.h>

#include "bfrag.cuh"
#include "common.cuh"
#include "kernels.h"
#include "model_dev.h"

#include <algorithm>

namespace cg = cooperative_groups;

namespace g4b {

constexpr int kAttnKeys = 64;  // keys per tile
constexpr int kAttnRows = 16;  // query rows per CTA (the MMA's M)
constexpr int kAttnWarps = 8;
constexpr int kAttnThreads = kAttnWarps * 32;
constexpr int kPStride = kAttnKeys + 8;  // halves per P row (conflict-free ldmatrix)
constexpr int kSStride = kAttnKeys + 4;  // floats per S row
constexpr float kPScale = 16384.0f;      // P is split after scaling by 2^14

constexpr int kMaxSplits = 16;  // largest cluster (non-portable size; B200 allows 16)

template <bool BF16>
struct AttnTypes;
template <>
struct AttnTypes<false> {
    static constexpr int kTerms = 2;
    static __device__ __forceinline__ uint16_t to_bits(float x) { return __half_as_ushort(__float2half_rn(x)); }
    static __device__ __forceinline__ float from_bits(uint16_t b) { return __half2float(__ushort_as_half(b)); }
};
template <>
struct AttnTypes<true> {
    // Two bf16 terms carry 16 significant bits of the query and of P: a relative error below
    // 2^-16, far inside the pass's tolerance, for a third fewer MMAs than three terms
    // (a 6-layer 31B pass at 30 000 cached keys: M = 9 1.67 -> 1.61 ms, M = 128 8.99 -> 8.39 ms).
    static constexpr int kTerms = 2;
    static __device__ __forceinline__ uint16_t to_bits(float x) {
        return __bfloat16_as_ushort(__float2bfloat16_rn(x));
    }
    static __device__ __forceinline__ float from_bits(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }
};

template <bool BF16>
__device__ __forceinline__ void mma_tc(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    if constexpr (BF16) {
        asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    } else {
        asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
    const uint32_t s = (uint32_t)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(s));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
    const uint32_t s = (uint32_t)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(s));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t& r0, uint32_t& r1, const void* p) {
    const uint32_t s = (uint32_t)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(s));
}
__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
// The float2 at shared-memory address `addr` of cluster CTA `rank` (distributed shared memory).
__device__ __forceinline__ float2 ld_cluster_f2(uint32_t addr, int rank) {
    uint32_t ra;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(addr), "r"(rank));
    float2 v;
    asm volatile("ld.shared::cluster.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(ra) : "memory");
    return v;
}
__device__ __forceinline__ void cp16(void* smem, const void* gmem) {
    const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem));
}

// Shared memory plan (KS = hd + 8 halves per Q/K/V row: conflict-free ldmatrix rows).
struct AttnSmem {
    uint16_t* q;     // [terms][16][KS]
    uint16_t* k;     // [64][KS]
    uint16_t* v;     // [64][KS]
    uint16_t* p;     // [terms][16][kPStride]
    float* s;        // [16][kSStride]
    float* corr;     // [16]
    float* qscale;   // [16] 2^-e of the row's query scaling
    float2* ml;      // [16] {running max, running sum}
    float* o;        // [16][hd] partial output after the key loop (aliases the K/V tile)
};

inline size_t attn_smem_bytes(int hd, int terms) {
    const size_t ks = hd + 8;
    return (size_t)terms * kAttnRows * ks * 2 + 2 * (size_t)kAttnKeys * ks * 2 +
           (size_t)terms * kAttnRows * kPStride * 2 + kAttnRows * kSStride * 4 + kAttnRows * 4 * 2 + kAttnRows * 8;
}

__device__ __forceinline__ AttnSmem attn_smem(unsigned char* raw, int hd, int terms) {
    AttnSmem s;
    const int ks = hd + 8;
    uint16_t* h = reinterpret_cast<uint16_t*>(raw);
    s.q = h;
    h += terms * kAttnRows * ks;
    s.k = h;
    s.v = h + kAttnKeys * ks;
    s.o = reinterpret_cast<float*>(h);  // 16 * hd * 4 bytes <= 2 * 64 * ks * 2
    h += 2 * kAttnKeys * ks;
    s.p = h;
    h += terms * kAttnRows * kPStride;
    s.s = reinterpret_cast<float*>(h);
    s.corr = s.s + kAttnRows * kSStride;
    s.qscale = s.corr + kAttnRows;
    s.ml = reinterpret_cast<float2*>(s.qscale + kAttnRows);
    return s;
}

template <bool BF16, int HD>
__global__ void __launch_bounds__(kAttnThreads, HD <= 256 ? 2 : 1) attention_kernel(AttnArgs a, void* bfrag) {
    using Ty = AttnTypes<BF16>;
    constexpr int kTerms = Ty::kTerms;
    constexpr int KS = HD + 8;
    constexpr int kColsPerWarp = HD / kAttnWarps;  // PV output columns per warp
    constexpr int kNT = kColsPerWarp / 8;          // PV n-tiles per warp
    constexpr int kChunks = HD / 8;                // 16-byte chunks per K/V row
    constexpr int kKeyStep = kAttnThreads / kChunks;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ __half stage[kAttnWarps][128];
    cg::cluster_group cluster = cg::this_cluster();
    AttnSmem sm = attn_smem(smem_raw, HD, kTerms);

    pdl_launch_dependents();
    const int split = (int)cluster.block_rank();
    const int nsplit = (int)cluster.num_blocks();
    const int kvh_i = blockIdx.y, chunk = blockIdx.z;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t4 = lane & 3;
    const int gqa = a.qh / a.kvh;
    const int R = a.M * gqa;
    const int base = a.sp->base_pos;

    // Key range of this chunk's rows (the union of their causal spans), then this split's share.
    const int m_first = (chunk * kAttnRows) / gqa, m_last = min(a.M - 1, (chunk * kAttnRows + kAttnRows - 1) / gqa);
    const int kmin = a.window ? max(0, base + m_first + 1 - a.window) : 0;
    const int kmax = base + m_last + 1;
    const int per = (kmax - kmin + nsplit - 1) / nsplit;
    const int ks = kmin + split * per, ke = min(kmax, ks + per);

    // Each thread copies one 16-byte column chunk c8 of keys j0, j0 + kKeyStep, ...
    const int c8 = threadIdx.x % kChunks, j0 = threadIdx.x / kChunks;
    const size_t head_off = (size_t)kvh_i * HD + c8 * 8;
    // K and V tiles stream as separate cp.async groups so each overlaps the other's use: K of
    // tile t+1 loads during the softmax and P V of tile t, V of tile t+1 during Q K^T of t+1.
    // load_half copies the tile's keys at positions [plo, phi) and zero-fills the slots past
    // the range (P = 0 there meets finite V); the caller commits the group.
    auto load_half = [&](int t0, const uint16_t* ring, uint16_t* dst, int plo, int phi) {
        const int nt = min(kAttnKeys, ke - t0);
        const int slot0 = t0 % a.cap;
        for (int j = j0; j < kAttnKeys; j += kKeyStep) {
            uint16_t* d = dst + j * KS + c8 * 8;
            if (j < nt) {
                if (t0 + j < plo || t0 + j >= phi) continue;
                int slot = slot0 + j;
                if (slot >= a.cap) slot %= a.cap;
                cp16(d, ring + (size_t)slot * a.kvh * HD + head_off);
            } else if (plo == kmin) {
                *reinterpret_cast<uint4*>(d) = make_uint4(0, 0, 0, 0);
            }
        }
    };
    auto commit = [] { asm volatile("cp.async.commit_group;" ::: "memory"); };
    // The first tile's keys from earlier passes are fetched before waiting on the producer
    // (the Q/K/V epilogue). Nothing in this pass changes them or base_pos: base_pos is written
    // only by a pass's last kernel (head_finalize), every pass starts with a kernel launched
    // without programmatic overlap, and this pass rewrites only the ring slots of positions
    // base.. (a sliding ring keeps window + max rows slots, so those never alias a key a row
    // still needs). The keys at base.. and the query rows are read after the wait. A prefill
    // chunk (two waves of CTAs, several tiles each) keeps the plain order, in which Q K^T of the
    // first tile waits for K alone.
    const int early = a.M > kMaxM ? kmin : base;  // keys [kmin, early) are fetched early
    if (ks < ke) {
        load_half(ks, a.k_ring, sm.k, kmin, early);
        load_half(ks, a.v_ring, sm.v, kmin, early);
    }
    pdl_wait();
    if (ks < ke) {
        load_half(ks, a.k_ring, sm.k, early, kmax);
        commit();
        load_half(ks, a.v_ring, sm.v, early, kmax);
        commit();
    }

    // Stage the query rows: warp w takes rows 2w, 2w+1. Scaling by 2^(15-e) puts the row's
    // max |q| in [2^14, 2^15); the scaled row is then split into terms of the MMA type.
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
        const int r = warp * 2 + rr;
        const int qr = chunk * kAttnRows + r;
        float x[HD / 32];
        float amax = 0.f;
        const float* src = nullptr;
        if (qr < R) {
            const int m = qr / gqa, qhead = kvh_i * gqa + qr % gqa;
            src = a.q + ((size_t)m * a.qh + qhead) * HD;
        }
#pragma unroll
        for (int j = 0; j < HD / 32; ++j) {
            x[j] = src ? src[lane + 32 * j] : 0.f;
            amax = fmaxf(amax, fabsf(x[j]));
        }
        amax = warp_max(amax);
        int e = 0;
        frexpf(amax, &e);
        const float sc = amax > 0.f ? ldexpf(1.0f, 15 - e) : 1.0f;
        if (lane == 0) sm.qscale[r] = amax > 0.f ? ldexpf(1.0f, e - 15) : 1.0f;
#pragma unroll
        for (int j = 0; j < HD / 32; ++j) {
            float rem = x[j] * sc;
#pragma unroll
            for (int tt = 0; tt < kTerms; ++tt) {
                const uint16_t b = Ty::to_bits(rem);
                sm.q[(tt * kAttnRows + r) * KS + lane + 32 * j] = b;
                rem -= Ty::from_bits(b);
            }
        }
    }
    // head_dim 512: Q K^T is split by head dimension instead of by key. Warp w keeps its 64-dim
    // slice of the query terms in registers for the whole key loop and multiplies it by the
    // same slice of all 64 keys of a tile; the eight partial score tiles are then added in
    // shared memory (in the Q staging buffer, free once the slices are in registers). Each
    // tile's K is read from shared memory once instead of the query once per warp.
    constexpr bool kSplitDims = HD == 512;
    constexpr int kDimsPerWarp = HD / kAttnWarps;
    uint32_t qf[kSplitDims ? kTerms : 1][kSplitDims ? kDimsPerWarp / 16 : 1][4];
    float* sp = reinterpret_cast<float*>(sm.q);  // [warp][16 rows][64 keys], column-swizzled
    auto sp_at = [&](int w, int row, int key) { return sp + (w * kAttnRows + row) * kAttnKeys + (key ^ ((row & 7) << 3)); };
    if constexpr (kSplitDims) {
        static_assert((size_t)kAttnWarps * kAttnRows * kAttnKeys * 4 <= (size_t)2 * kAttnRows * (HD + 8) * 2,
                      "partial scores must fit the query staging buffer");
        __syncthreads();  // the staged query terms are visible
        const uint16_t* qb = sm.q + (lane & 15) * KS + warp * kDimsPerWarp + (lane >> 4) * 8;
#pragma unroll
        for (int tt = 0; tt < kTerms; ++tt)
#pragma unroll
            for (int kk = 0; kk < kDimsPerWarp / 16; ++kk) ldsm_x4(qf[tt][kk], qb + tt * kAttnRows * KS + kk * 16);
        __syncthreads();  // every warp holds its slice: the buffer now takes partial scores
    }
    // Softmax state: warp w owns rows 2w, 2w+1 (every lane keeps the same copy).
    float m_run[2], l_run[2];
    int row_lo[2], row_hi[2];
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
        m_run[rr] = -INFINITY;
        l_run[rr] = 0.f;
        const int qr = chunk * kAttnRows + warp * 2 + rr;
        if (qr < R) {
            const int end = base + qr / gqa + 1;
            row_hi[rr] = end;
            row_lo[rr] = a.window ? max(0, end - a.window) : 0;
        } else {
            row_hi[rr] = row_lo[rr] = 0;  // empty span: the row stays masked
        }
    }
    float acc[kNT][4];
#pragma unroll
    for (int n = 0; n < kNT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;

    for (int t0 = ks; t0 < ke; t0 += kAttnKeys) {
        const bool more = t0 + kAttnKeys < ke;
        asm volatile("cp.async.wait_group 1;" ::: "memory");  // K of tile t0 (V may still land)
        __syncthreads();  // K of tile t0 (and the staged q) visible

        if constexpr (kSplitDims) {
            // Partial S[16 rows][64 keys] over this warp's 64 dimensions.
            float sj[kAttnKeys / 8][4];
            const uint16_t* kb = sm.k + (lane & 7) * KS + warp * kDimsPerWarp + (lane >> 3) * 8;
#pragma unroll
            for (int j = 0; j < kAttnKeys / 8; ++j) {
                sj[j][0] = sj[j][1] = sj[j][2] = sj[j][3] = 0.f;
#pragma unroll
                for (int kh = 0; kh < kDimsPerWarp / 32; ++kh) {
                    uint32_t b[4];
                    ldsm_x4(b, kb + (8 * j) * KS + kh * 32);  // dims +0..15 and +16..31 of keys 8j..8j+7
#pragma unroll
                    for (int tt = 0; tt < kTerms; ++tt) {
                        mma_tc<BF16>(sj[j], qf[tt][2 * kh], b[0], b[1]);
                        mma_tc<BF16>(sj[j], qf[tt][2 * kh + 1], b[2], b[3]);
                    }
                }
                *reinterpret_cast<float2*>(sp_at(warp, g, 8 * j + 2 * t4)) = make_float2(sj[j][0], sj[j][1]);
                *reinterpret_cast<float2*>(sp_at(warp, g + 8, 8 * j + 2 * t4)) = make_float2(sj[j][2], sj[j][3]);
            }
        } else {
        // S[16 rows][keys 8w..8w+7] = sum over terms of Q_t K^T.
            float s[4] = {0.f, 0.f, 0.f, 0.f};
            const uint16_t* kb = sm.k + (warp * 8 + (lane & 7)) * KS + (lane >> 3) * 8;
            const uint16_t* qb = sm.q + (lane & 15) * KS + (lane >> 4) * 8;
#pragma unroll 4
            for (int k0 = 0; k0 < HD; k0 += 32) {
                uint32_t b[4];
                ldsm_x4(b, kb + k0);  // k-steps k0 and k0 + 16
#pragma unroll
                for (int tt = 0; tt < kTerms; ++tt) {
                    uint32_t q0[4], q1[4];
                    ldsm_x4(q0, qb + tt * kAttnRows * KS + k0);
                    ldsm_x4(q1, qb + tt * kAttnRows * KS + k0 + 16);
                    mma_tc<BF16>(s, q0, b[0], b[1]);
                    mma_tc<BF16>(s, q1, b[2], b[3]);
                }
            }
            float* sr = sm.s + g * kSStride + warp * 8 + 2 * t4;
            sr[0] = s[0];
            sr[1] = s[1];
            sr[8 * kSStride] = s[2];
            sr[8 * kSStride + 1] = s[3];
        }
        __syncthreads();  // every warp is done with K of tile t0
        if (more) load_half(t0 + kAttnKeys, a.k_ring, sm.k, kmin, kmax);
        commit();  // (an empty group past the last tile keeps the group count uniform)

        // Online softmax: keys lane and lane + 32 of the tile.
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            const int r = warp * 2 + rr;
            float sc[2];
            bool valid[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int kl = lane + 32 * h, tk = t0 + kl;
                valid[h] = tk < ke && tk >= row_lo[rr] && tk < row_hi[rr];
                float sv;
                if constexpr (kSplitDims) {
                    sv = 0.f;
#pragma unroll
                    for (int w = 0; w < kAttnWarps; ++w) sv += *sp_at(w, r, kl);
                } else {
                    sv = sm.s[r * kSStride + kl];
                }
                sc[h] = valid[h] ? sv * sm.qscale[r] * a.scale : -INFINITY;
            }
            const float m_new = fmaxf(m_run[rr], warp_max(fmaxf(sc[0], sc[1])));
            float p[2] = {0.f, 0.f}, corr = 1.f;
            if (m_new != -INFINITY) {
                p[0] = valid[0] ? expf(sc[0] - m_new) : 0.f;
                p[1] = valid[1] ? expf(sc[1] - m_new) : 0.f;
                corr = expf(m_run[rr] - m_new);  // 0 on the first contributing tile
            }
            l_run[rr] = l_run[rr] * corr + warp_sum(p[0] + p[1]);
            m_run[rr] = m_new;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float rem = p[h] * kPScale;
#pragma unroll
                for (int tt = 0; tt < kTerms; ++tt) {
                    const uint16_t b = Ty::to_bits(rem);
                    sm.p[(tt * kAttnRows + r) * kPStride + lane + 32 * h] = b;
                    rem -= Ty::from_bits(b);
                }
            }
            if (lane == 0) sm.corr[r] = corr;
        }
        asm volatile("cp.async.wait_group 1;" ::: "memory");  // V of tile t0 (K of t0+1 may still land)
        __syncthreads();  // P, the corrections and V of tile t0 visible

        // O[16][warp's columns] = O * corr + sum over terms of P_t V.
        {
            const float c0 = sm.corr[g], c1 = sm.corr[g + 8];
#pragma unroll
            for (int n = 0; n < kNT; ++n) {
                acc[n][0] *= c0;
                acc[n][1] *= c0;
                acc[n][2] *= c1;
                acc[n][3] *= c1;
            }
#pragma unroll
            for (int kk = 0; kk < kAttnKeys; kk += 16) {
                uint32_t pa[kTerms][4];
#pragma unroll
                for (int tt = 0; tt < kTerms; ++tt)
                    ldsm_x4(pa[tt], sm.p + (tt * kAttnRows + (lane & 15)) * kPStride + kk + (lane >> 4) * 8);
                if constexpr (kNT == 1) {
                    uint32_t b0, b1;
                    ldsm_x2_t(b0, b1, sm.v + (kk + (lane & 7) + ((lane >> 3) & 1) * 8) * KS + warp * kColsPerWarp);
#pragma unroll
                    for (int tt = 0; tt < kTerms; ++tt) mma_tc<BF16>(acc[0], pa[tt], b0, b1);
                } else {
                    const uint16_t* vb = sm.v + (kk + (lane & 7) + ((lane >> 3) & 1) * 8) * KS + warp * kColsPerWarp +
                                         (lane >> 4) * 8;
#pragma unroll
                    for (int n = 0; n < kNT; n += 2) {
                        uint32_t b[4];
                        ldsm_x4_t(b, vb + n * 8);  // n-tiles n and n + 1
#pragma unroll
                        for (int tt = 0; tt < kTerms; ++tt) {
                            mma_tc<BF16>(acc[n], pa[tt], b[0], b[1]);
                            mma_tc<BF16>(acc[n + 1], pa[tt], b[2], b[3]);
                        }
                    }
                }
            }
        }
        __syncthreads();  // every warp is done with V of tile t0
        if (more) {
            load_half(t0 + kAttnKeys, a.v_ring, sm.v, kmin, kmax);
            commit();
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();  // every warp is done with the K/V tile: sm.o may overwrite it

    // This split's partial result: unnormalised O (P's 2^14 scale removed) and {m, l}.
#pragma unroll
    for (int n = 0; n < kNT; ++n) {
        const int col = warp * kColsPerWarp + n * 8 + 2 * t4;
        *reinterpret_cast<float2*>(sm.o + g * HD + col) = make_float2(acc[n][0] / kPScale, acc[n][1] / kPScale);
        *reinterpret_cast<float2*>(sm.o + (g + 8) * HD + col) = make_float2(acc[n][2] / kPScale, acc[n][3] / kPScale);
    }
    if (lane == 0)
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) sm.ml[warp * 2 + rr] = make_float2(m_run[rr], l_run[rr]);
    cluster.sync();

    // Combine across the cluster: out = sum_s e^(m_s - M) O_s / sum_s e^(m_s - M) l_s, one warp
    // per (row, 64-column group), the items spread over the cluster's CTAs. Each warp loads
    // every split's {m, l} and partial output before combining, so the remote reads overlap.
    constexpr int kGroups = HD / 64;
    const int K = a.qh * HD;
    const BFragView bv = bfrag_view(bfrag, (K + 127) / 128 * 128, a.M);
    // Prefill rows (wide layout) take one static scale per row: every output is a convex
    // combination of cached V rows, and V is RMS-normalised without a weight, so
    // |o| <= max |v| <= sqrt(head_dim) (times the cache's rounding, well inside 1.01).
    const bool wide = a.M > kMaxM;
    const float wide_e = wide_row_scale(sqrtf((float)HD) * 1.01f), wide_inv = 1.0f / wide_e;
    for (int w = split * kAttnWarps + warp; w < kAttnRows * kGroups; w += nsplit * kAttnWarps) {
        const int r = w / kGroups, gi = w % kGroups;
        const int qr = chunk * kAttnRows + r;
        if (qr >= R) continue;  // warp-uniform
        // Every split's {m, l} and partial output in one round of remote loads (32-bit cluster
        // addresses keep the 32 loads in flight within the register budget).
        float2 ml[kMaxSplits], op[kMaxSplits];
        const uint32_t ml_addr = smem_addr(sm.ml + r), o_addr = smem_addr(sm.o + r * HD + gi * 64 + 2 * lane);
#pragma unroll
        for (int s = 0; s < kMaxSplits; ++s) {
            ml[s] = make_float2(-INFINITY, 0.f);
            op[s] = make_float2(0.f, 0.f);
            if (s < nsplit) {
                ml[s] = ld_cluster_f2(ml_addr, s);
                op[s] = ld_cluster_f2(o_addr, s);
            }
        }
        float mx = -INFINITY;
#pragma unroll
        for (int s = 0; s < kMaxSplits; ++s) mx = fmaxf(mx, ml[s].x);
        float n0 = 0.f, n1 = 0.f, den = 0.f;
#pragma unroll
        for (int s = 0; s < kMaxSplits; ++s) {
            if (s >= nsplit || ml[s].y <= 0.f) continue;
            const float wgt = expf(ml[s].x - mx);
            n0 += wgt * op[s].x;
            n1 += wgt * op[s].y;
            den += wgt * ml[s].y;
        }
        const float inv = den > 0.f ? 1.0f / den : 0.f;
        const int m = qr / gqa, qhead = kvh_i * gqa + qr % gqa;
        if (wide) {
            wide_store_group(bv, m, (qhead * HD) / 64 + gi, n0 * inv, n1 * inv, wide_inv);
            if (lane == 0 && qhead == 0 && gi == 0) bv.erow[m] = wide_e;
        } else {
            bfrag_store_group(bv, a.M, m, (qhead * HD) / 64 + gi, n0 * inv, n1 * inv, stage[warp]);
        }
    }
    // A K that is not a multiple of 128 leaves one pad group per row: zero fragments.
    if ((K & 127) && blockIdx.y == 0 && blockIdx.z == 0 && split == 0)
        for (int m = warp; m < a.M; m += kAttnWarps) {
            if (wide) wide_store_group(bv, m, K / 64, 0.f, 0.f, wide_inv);
            else bfrag_store_group(bv, a.M, m, K / 64, 0.f, 0.f, stage[warp]);
        }
    cluster.sync();  // keep every CTA's shared memory alive until all remote reads are done
}

template <bool BF16, int HD>
static cudaLaunchConfig_t attn_config(const AttnArgs& a, int splits, cudaStream_t st, cudaLaunchAttribute* attr,
                                      bool pdl) {
    const int chunks = (a.M * (a.qh / a.kvh) + kAttnRows - 1) / kAttnRows;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(splits, a.kvh, chunks);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = attn_smem_bytes(HD, 2);
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    return cfg;
}

// Largest cluster size (key splits) whose clusters all fit on the GPU at once, so the launch is
// one wave; the occupancy query is made once per (kernel, size). Sizes above 8 are non-portable
// cluster sizes B200 allows.
constexpr int kSplitSizes[] = {16, 12, 8, 7, 6, 5, 4, 3, 2, 1};
constexpr int kNumSplitSizes = sizeof(kSplitSizes) / sizeof(kSplitSizes[0]);
template <bool BF16, int HD>
static int attn_splits(int clusters) {
    static int max_active[kNumSplitSizes];
    static bool queried = false;
    if (!queried) {
        for (int i = 0; i < kNumSplitSizes; ++i) {
            AttnArgs probe{};
            probe.M = 1;
            probe.qh = probe.kvh = 1;
            cudaLaunchAttribute attr[2];
            cudaLaunchConfig_t cfg = attn_config<BF16, HD>(probe, kSplitSizes[i], nullptr, attr, false);
            int n = 0;
            if (cudaOccupancyMaxActiveClusters(&n, attention_kernel<BF16, HD>, &cfg) != cudaSuccess) {
                cudaGetLastError();
                n = 0;
            }
            max_active[i] = n;
        }
        queried = true;
    }
    for (int i = 0; i < kNumSplitSizes; ++i)
        if (max_active[i] >= clusters) return kSplitSizes[i];
    return 1;
}

template <bool BF16, int HD>
static cudaError_t launch_attn(const AttnArgs& a, void* bfrag, cudaStream_t st, bool pdl) {
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(attention_kernel<BF16, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)attn_smem_bytes(HD, 2));
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(attention_kernel<BF16, HD>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    const int chunks = (a.M * (a.qh / a.kvh) + kAttnRows - 1) / kAttnRows;
    // A verify pass has few clusters: split the keys as widely as one wave allows. A prefill
    // chunk has hundreds of clusters already, so its keys are split in two only, which keeps the
    // per-CTA loops long and the cross-CTA combine cheap.
    int splits = a.M > kMaxM ? 2 : attn_splits<BF16, HD>(a.kvh * chunks);
    // A sliding layer's key range is bounded by its window whatever the context, so when there
    // are clusters enough to fill the GPU (8 or more), 8 splits already leave each CTA at most
    // two 64-key tiles of a 1024-key window; more only add combine work (measured: 31B 5-row
    // verify pass 5.85 -> 5.78 ms, long-context passes unchanged). With few clusters (the
    // drafter's single KV head) the wide split stays: capped, a 3-row drafter pass went 1.44 ->
    // 1.53 ms. Full-attention layers keep the widest split that fits one wave.
    if (a.window > 0 && a.window <= 1024 && a.kvh * chunks >= 8) splits = std::min(splits, 8);
    cudaLaunchAttribute attr[2];
    cudaLaunchConfig_t cfg = attn_config<BF16, HD>(a, splits, st, attr, pdl);
    return cudaLaunchKernelEx(&cfg, attention_kernel<BF16, HD>, a, bfrag);
}

template <int HD>
static cudaError_t launch_hd(const AttnArgs& a, void* bfrag, cudaStream_t st, bool pdl) {
    return a.kv_bf16 ? launch_attn<true, HD>(a, bfrag, st, pdl) : launch_attn<false, HD>(a, bfrag, st, pdl);
}

}  // namespace g4b

using namespace g4b;

cudaError_t g4b_attention(const AttnArgs& a, void* bfrag, cudaStream_t st, bool pdl) {
    if (a.kvh < 1 || a.qh % a.kvh || a.M < 1 || a.M > kPrefillRows) return cudaErrorInvalidValue;
    switch (a.hd) {
        case 64: return launch_hd<64>(a, bfrag, st, pdl);
        case 128: return launch_hd<128>(a, bfrag, st, pdl);
        case 256: return launch_hd<256>(a, bfrag, st, pdl);
        case 512: return launch_hd<512>(a, bfrag, st, pdl);
        default: return cudaErrorInvalidValue;
    }
}
