// Multi-row GQA attention over the KV ring -- Attention.hlsl (shaders/Attention.hlsl:65-179)
// rebuilt so the KV cache is read ONCE per KV head for all M verify rows and all of that
// head's query heads (the reference dispatches one group per (row, query head), re-reading
// the cache M * q_heads/kv_heads times).
//
// Grid: one thread-block cluster of kSplits CTAs per (KV head, chunk of 16 query rows); CTA r
// of the cluster takes the r-th share of the batch's key range. Per 32-key tile (K and V
// double-buffered in shared memory by cp.async):
//   * S = Q K^T on the tensor cores (mma.sync m16n8k16, fp32 accumulate). The cached K is
//     exact in the MMA's input type (FP16, or bf16 in long-context mode); the fp32 query is
//     split into 2 (FP16) or 3 (bf16) terms q = q1 + q2 (+ q3) after a power-of-two row
//     scaling, so the scores carry the fp32 query's precision. Warp w computes keys 8w..8w+7;
//   * an online softmax per row (running max / sum in fp32, exp of the fp32 scores);
//   * O += P V on the tensor cores with P (scaled by 2^14) split the same way; warp w owns
//     columns [w*hd/4, (w+1)*hd/4) of the output.
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

constexpr int kAttnKeys = 32;  // keys per tile
constexpr int kAttnRows = 16;  // query rows per CTA (the MMA's M)
constexpr int kAttnWarps = 4;
constexpr int kAttnThreads = kAttnWarps * 32;
constexpr int kSplits = 8;               // CTAs per cluster = key splits
constexpr int kPStride = kAttnKeys + 8;  // halves per P row (conflict-free ldmatrix)
constexpr int kSStride = kAttnKeys + 4;  // floats per S row
constexpr float kPScale = 16384.0f;      // P is split after scaling by 2^14

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
    static constexpr int kTerms = 3;
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
__device__ __forceinline__ void cp16(void* smem, const void* gmem) {
    const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem));
}

// Shared memory plan (KS = hd + 8 halves per Q/K/V row: conflict-free ldmatrix rows).
struct AttnSmem {
    uint16_t* q;     // [terms][16][KS]
    uint16_t* kv;    // 2 buffers x {K [32][KS], V [32][KS]}
    uint16_t* p;     // [terms][16][kPStride]
    float* s;        // [16][kSStride]
    float* corr;     // [16]
    float* qscale;   // [16] 2^-e of the row's query scaling
    float2* ml;      // [16] {running max, running sum}
    float* o;        // [16][hd] partial output after the key loop (aliases the K/V tiles)
};

inline size_t attn_smem_bytes(int hd, int terms) {
    const size_t ks = hd + 8;
    return (size_t)terms * kAttnRows * ks * 2 + 4 * (size_t)kAttnKeys * ks * 2 +
           (size_t)terms * kAttnRows * kPStride * 2 + kAttnRows * kSStride * 4 + kAttnRows * 4 * 2 + kAttnRows * 8;
}

__device__ __forceinline__ AttnSmem attn_smem(unsigned char* raw, int hd, int terms) {
    AttnSmem s;
    const int ks = hd + 8;
    uint16_t* h = reinterpret_cast<uint16_t*>(raw);
    s.q = h;
    h += terms * kAttnRows * ks;
    s.kv = h;
    s.o = reinterpret_cast<float*>(h);  // 16 * hd * 4 bytes <= 4 * 32 * ks * 2
    h += 4 * kAttnKeys * ks;
    s.p = h;
    h += terms * kAttnRows * kPStride;
    s.s = reinterpret_cast<float*>(h);
    s.corr = s.s + kAttnRows * kSStride;
    s.qscale = s.corr + kAttnRows;
    s.ml = reinterpret_cast<float2*>(s.qscale + kAttnRows);
    return s;
}

template <bool BF16, int HD>
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(AttnArgs a, void* bfrag) {
    using Ty = AttnTypes<BF16>;
    constexpr int kTerms = Ty::kTerms;
    constexpr int KS = HD + 8;
    constexpr int kColsPerWarp = HD / kAttnWarps;  // PV output columns per warp
    constexpr int kNT = kColsPerWarp / 8;          // PV n-tiles per warp
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ __half stage[kAttnWarps][128];
    cg::cluster_group cluster = cg::this_cluster();
    AttnSmem sm = attn_smem(smem_raw, HD, kTerms);

    pdl_enter();
    const int split = (int)cluster.block_rank();
    const int kvh_i = blockIdx.y, chunk = blockIdx.z;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t4 = lane & 3;
    const int gqa = a.qh / a.kvh;
    const int R = a.M * gqa;
    const int base = a.sp->base_pos;

    // Key range of the whole batch, then this split's share.
    const int kmin = a.window ? max(0, base + 1 - a.window) : 0;
    const int kmax = base + a.M;
    const int per = (kmax - kmin + kSplits - 1) / kSplits;
    const int ks = kmin + split * per, ke = min(kmax, ks + per);

    auto load_tile = [&](int t0, int buf) {
        const int nt = min(kAttnKeys, ke - t0);
        for (int i = threadIdx.x; i < kAttnKeys * (HD / 8); i += kAttnThreads) {
            const int j = i / (HD / 8), c8 = i % (HD / 8);
            uint16_t* kd = sm.kv + (2 * buf * kAttnKeys + j) * KS + c8 * 8;
            uint16_t* vd = kd + kAttnKeys * KS;
            if (j < nt) {
                const size_t src = ((size_t)((t0 + j) % a.cap) * a.kvh + kvh_i) * HD + c8 * 8;
                cp16(kd, a.k_ring + src);
                cp16(vd, a.v_ring + src);
            } else {  // keys past the range: zeros, so P = 0 meets finite V
                *reinterpret_cast<uint4*>(kd) = make_uint4(0, 0, 0, 0);
                *reinterpret_cast<uint4*>(vd) = make_uint4(0, 0, 0, 0);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    if (ks < ke) load_tile(ks, 0);

    // Stage the query rows: warp w takes rows 4w..4w+3. Scaling by 2^(15-e) puts the row's
    // max |q| in [2^14, 2^15); the scaled row is then split into terms of the MMA type.
    for (int rr = 0; rr < 4; ++rr) {
        const int r = warp * 4 + rr;
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
    // Softmax state: warp w owns rows 4w..4w+3 (every lane keeps the same copy).
    float m_run[4], l_run[4];
    int row_lo[4], row_hi[4];
#pragma unroll
    for (int rr = 0; rr < 4; ++rr) {
        m_run[rr] = -INFINITY;
        l_run[rr] = 0.f;
        const int qr = chunk * kAttnRows + warp * 4 + rr;
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

    int buf = 0;
    for (int t0 = ks; t0 < ke; t0 += kAttnKeys, buf ^= 1) {
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        __syncthreads();  // tile t0 (and the staged q) visible; every warp is past the last PV
        if (t0 + kAttnKeys < ke) load_tile(t0 + kAttnKeys, buf ^ 1);

        // S[16 rows][keys 8w..8w+7] = sum over terms of Q_t K^T.
        {
            float s[4] = {0.f, 0.f, 0.f, 0.f};
            const uint16_t* kb = sm.kv + (2 * buf * kAttnKeys + warp * 8 + (lane & 7)) * KS + (lane >> 3) * 8;
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
        __syncthreads();

        // Online softmax: lane = key of the tile.
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) {
            const int r = warp * 4 + rr;
            const int tk = t0 + lane;
            const bool valid = lane < ke - t0 && tk >= row_lo[rr] && tk < row_hi[rr];
            const float sc = valid ? sm.s[r * kSStride + lane] * sm.qscale[r] * a.scale : -INFINITY;
            const float m_new = fmaxf(m_run[rr], warp_max(sc));
            float p = 0.f, corr = 1.f;
            if (m_new != -INFINITY) {
                p = valid ? expf(sc - m_new) : 0.f;
                corr = expf(m_run[rr] - m_new);  // 0 on the first contributing tile
            }
            l_run[rr] = l_run[rr] * corr + warp_sum(p);
            m_run[rr] = m_new;
            float rem = p * kPScale;
#pragma unroll
            for (int tt = 0; tt < kTerms; ++tt) {
                const uint16_t b = Ty::to_bits(rem);
                sm.p[(tt * kAttnRows + r) * kPStride + lane] = b;
                rem -= Ty::from_bits(b);
            }
            if (lane == 0) sm.corr[r] = corr;
        }
        __syncthreads();

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
                const uint16_t* vb = sm.kv + ((2 * buf + 1) * kAttnKeys + kk + (lane & 7) + ((lane >> 3) & 1) * 8) * KS +
                                     warp * kColsPerWarp + (lane >> 4) * 8;
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
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();  // every warp is done with the K/V tiles: sm.o may overwrite them

    // This split's partial result: unnormalised O (P's 2^14 scale removed) and {m, l}.
#pragma unroll
    for (int n = 0; n < kNT; ++n) {
        const int col = warp * kColsPerWarp + n * 8 + 2 * t4;
        *reinterpret_cast<float2*>(sm.o + g * HD + col) = make_float2(acc[n][0] / kPScale, acc[n][1] / kPScale);
        *reinterpret_cast<float2*>(sm.o + (g + 8) * HD + col) = make_float2(acc[n][2] / kPScale, acc[n][3] / kPScale);
    }
    if (lane == 0)
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) sm.ml[warp * 4 + rr] = make_float2(m_run[rr], l_run[rr]);
    cluster.sync();

    // Combine across the cluster: out = sum_s e^(m_s - M) O_s / sum_s e^(m_s - M) l_s, one warp
    // per (row, 64-column group), the items spread over the cluster's CTAs.
    constexpr int kGroups = HD / 64;
    const int K = a.qh * HD;
    const BFragView bv = bfrag_view(bfrag, (K + 127) / 128 * 128, a.M);
    for (int w = split * kAttnWarps + warp; w < kAttnRows * kGroups; w += kSplits * kAttnWarps) {
        const int r = w / kGroups, gi = w % kGroups;
        const int qr = chunk * kAttnRows + r;
        if (qr >= R) continue;  // warp-uniform
        float mx = -INFINITY;
        for (int s = 0; s < kSplits; ++s) mx = fmaxf(mx, cluster.map_shared_rank(sm.ml, s)[r].x);
        float n0 = 0.f, n1 = 0.f, den = 0.f;
        for (int s = 0; s < kSplits; ++s) {
            const float2 ml = cluster.map_shared_rank(sm.ml, s)[r];
            if (ml.y <= 0.f) continue;
            const float wgt = expf(ml.x - mx);
            const float2 op =
                *reinterpret_cast<const float2*>(cluster.map_shared_rank(sm.o, s) + r * HD + gi * 64 + 2 * lane);
            n0 += wgt * op.x;
            n1 += wgt * op.y;
            den += wgt * ml.y;
        }
        const float inv = den > 0.f ? 1.0f / den : 0.f;
        const int m = qr / gqa, qhead = kvh_i * gqa + qr % gqa;
        bfrag_store_group(bv, a.M, m, (qhead * HD) / 64 + gi, n0 * inv, n1 * inv, stage[warp]);
    }
    // A K that is not a multiple of 128 leaves one pad group per row: zero fragments.
    if ((K & 127) && blockIdx.y == 0 && blockIdx.z == 0 && split == 0)
        for (int m = warp; m < a.M; m += kAttnWarps) bfrag_store_group(bv, a.M, m, K / 64, 0.f, 0.f, stage[warp]);
    cluster.sync();  // keep every CTA's shared memory alive until all remote reads are done
}

template <bool BF16, int HD>
static cudaError_t launch_attn(const AttnArgs& a, void* bfrag, cudaStream_t st, bool pdl) {
    const size_t smem = attn_smem_bytes(HD, BF16 ? 3 : 2);
    static bool attr_set = false;
    if (!attr_set) {
        const cudaError_t e = cudaFuncSetAttribute(attention_kernel<BF16, HD>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    const int chunks = (a.M * (a.qh / a.kvh) + kAttnRows - 1) / kAttnRows;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kSplits, a.kvh, chunks);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kSplits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, attention_kernel<BF16, HD>, a, bfrag);
}

template <int HD>
static cudaError_t launch_hd(const AttnArgs& a, void* bfrag, cudaStream_t st, bool pdl) {
    return a.kv_bf16 ? launch_attn<true, HD>(a, bfrag, st, pdl) : launch_attn<false, HD>(a, bfrag, st, pdl);
}

}  // namespace g4b

using namespace g4b;

cudaError_t g4b_attention(const AttnArgs& a, void* bfrag, cudaStream_t st, bool pdl) {
    if (a.kvh < 1 || a.qh % a.kvh || a.M < 1 || a.M > kMaxM) return cudaErrorInvalidValue;
    switch (a.hd) {
        case 64: return launch_hd<64>(a, bfrag, st, pdl);
        case 128: return launch_hd<128>(a, bfrag, st, pdl);
        case 256: return launch_hd<256>(a, bfrag, st, pdl);
        case 512: return launch_hd<512>(a, bfrag, st, pdl);
        default: return cudaErrorInvalidValue;
    }
}
