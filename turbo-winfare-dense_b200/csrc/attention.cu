// Multi-row GQA attention over the KV ring -- Attention.hlsl (shaders/Attention.hlsl:65-179)
// rebuilt so the KV cache is read ONCE per KV head for all M verify rows and all of that
// head's query heads (the reference dispatches one group per (row, query head), re-reading
// the cache M * q_heads/kv_heads times).
//
// Grid: one thread-block cluster of kSplits CTAs per (KV head, chunk of 16 query rows); CTA
// r of the cluster takes the r-th share of the batch's key range. Each CTA streams 32-key
// tiles of K and V into shared memory (cp.async, double-buffered), each warp owns two query
// rows, scores are fp32 dot products of the fp32 query with the rounded K, and an online
// softmax (running max / sum) accumulates the unnormalised output. The cluster's partial
// results are then combined through distributed shared memory -- no global round trip --
// and written directly as the o-projection's B fragments.
//
// Row m of the batch sits at position base+m and sees keys [max(0, base+m+1-window),
// base+m+1) (all keys from 0 on full-attention layers): the reference's per-row causal span
// (shaders/Attention.hlsl:82-86). Scale is a parameter (1.0 for Gemma 4,
// src/cpu_reference.cpp:508-510).
#include <cooperative_groups.h>

#include "bfrag.cuh"
#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"
#include "model_dev.h"

#include <algorithm>

namespace cg = cooperative_groups;

namespace g4b {

constexpr int kAttnKeys = 32;    // keys per tile (one per lane)
constexpr int kAttnRows = 16;    // query rows per CTA (two per warp)
constexpr int kAttnThreads = 256;
constexpr int kSplits = 8;       // CTAs per cluster = key splits

__device__ __forceinline__ float2 kv_pair(uint32_t bits2, int bf16) {
    if (bf16) return make_float2(__uint_as_float(bits2 << 16), __uint_as_float(bits2 & 0xFFFF0000u));
    return __half22float2(*reinterpret_cast<const __half2*>(&bits2));
}

__device__ __forceinline__ void cp16(void* smem, const void* gmem) {
    const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem));
}

struct AttnSmem {
    float* q;        // [16][hd]; reused for this CTA's partial output after the key loop
    uint16_t* k[2];  // [32][hd + 8]
    uint16_t* v[2];  // [32][hd]
    float* p;        // [16][32]
    float2* ml;      // [16] running {max, sum}
};

__device__ __forceinline__ AttnSmem attn_smem(unsigned char* raw, int hd) {
    AttnSmem s;
    s.q = reinterpret_cast<float*>(raw);
    uint16_t* kv = reinterpret_cast<uint16_t*>(s.q + kAttnRows * hd);
    const int ktile = kAttnKeys * (hd + 8), vtile = kAttnKeys * hd;
    s.k[0] = kv;
    s.v[0] = kv + ktile;
    s.k[1] = kv + ktile + vtile;
    s.v[1] = kv + 2 * ktile + vtile;
    s.p = reinterpret_cast<float*>(kv + 2 * (ktile + vtile));
    s.ml = reinterpret_cast<float2*>(s.p + kAttnRows * kAttnKeys);
    return s;
}

__global__ void __launch_bounds__(kAttnThreads) attention_kernel(AttnArgs a, void* bfrag) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ __half stage[kAttnThreads / 32][128];
    cg::cluster_group cluster = cg::this_cluster();
    const int hd = a.hd;
    const int kstride = hd + 8;
    AttnSmem sm = attn_smem(smem_raw, hd);

    pdl_enter();
    const int split = (int)cluster.block_rank();
    const int kvh_i = blockIdx.y, chunk = blockIdx.z;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gqa = a.qh / a.kvh;
    const int R = a.M * gqa;
    const int base = a.sp->base_pos;

    // Stage this chunk's query rows.
    for (int i = threadIdx.x; i < kAttnRows * hd; i += kAttnThreads) {
        const int r = i / hd, d = i % hd;
        const int qr = chunk * kAttnRows + r;
        float v = 0.f;
        if (qr < R) {
            const int m = qr / gqa, qhead = kvh_i * gqa + qr % gqa;
            v = a.q[((size_t)m * a.qh + qhead) * hd + d];
        }
        sm.q[i] = v;
    }
    __syncthreads();  // q is complete before any warp reads it or (empty split) overwrites it

    // Key range of the whole batch, then this split's share.
    const int kmin = a.window ? max(0, base + 1 - a.window) : 0;
    const int kmax = base + a.M;
    const int per = (kmax - kmin + kSplits - 1) / kSplits;
    const int ks = kmin + split * per, ke = min(kmax, ks + per);

    int row_lo[2], row_hi[2];
    bool row_ok[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const int qr = chunk * kAttnRows + warp * 2 + j;
        row_ok[j] = qr < R;
        const int end = base + (row_ok[j] ? qr / gqa : 0) + 1;
        row_hi[j] = min(end, ke);
        row_lo[j] = max(a.window ? max(0, end - a.window) : 0, ks);
    }
    const int npair = hd / 64;  // dim pairs per lane: d = 2*lane + 64*i
    float o[2][8][2];
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int i = 0; i < 8; ++i) o[j][i][0] = o[j][i][1] = 0.f;
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};

    const int chunks_per_row = hd / 8;
    auto load_tile = [&](int t0, int buf) {
        const int nt = min(kAttnKeys, ke - t0);
        for (int i = threadIdx.x; i < kAttnKeys * chunks_per_row; i += kAttnThreads) {
            const int j = i / chunks_per_row, c8 = i % chunks_per_row;
            if (j < nt) {
                const size_t src = ((size_t)((t0 + j) % a.cap) * a.kvh + kvh_i) * hd + c8 * 8;
                cp16(sm.k[buf] + j * kstride + c8 * 8, a.k_ring + src);
                cp16(sm.v[buf] + j * hd + c8 * 8, a.v_ring + src);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };

    int buf = 0;
    if (ks < ke) load_tile(ks, 0);
    for (int t0 = ks; t0 < ke; t0 += kAttnKeys, buf ^= 1) {
        const int nt = min(kAttnKeys, ke - t0);
        // Prefetch the next tile into the other buffer, then wait for this one.
        if (t0 + kAttnKeys < ke) {
            load_tile(t0 + kAttnKeys, buf ^ 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();

        // Scores: lane = key, two rows per warp.
        float s[2] = {0.f, 0.f};
        const uint16_t* kr = sm.k[buf] + lane * kstride;
        for (int d = 0; d < hd; d += 8) {
            const uint4 kb = *reinterpret_cast<const uint4*>(kr + d);
            const float2 k01 = kv_pair(kb.x, a.kv_bf16), k23 = kv_pair(kb.y, a.kv_bf16);
            const float2 k45 = kv_pair(kb.z, a.kv_bf16), k67 = kv_pair(kb.w, a.kv_bf16);
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const float4 qa = *reinterpret_cast<const float4*>(sm.q + (warp * 2 + j) * hd + d);
                const float4 qb = *reinterpret_cast<const float4*>(sm.q + (warp * 2 + j) * hd + d + 4);
                s[j] += qa.x * k01.x + qa.y * k01.y + qa.z * k23.x + qa.w * k23.y + qb.x * k45.x + qb.y * k45.y +
                        qb.z * k67.x + qb.w * k67.y;
            }
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int t = t0 + lane;
            const bool valid = row_ok[j] && lane < nt && t >= row_lo[j] && t < row_hi[j];
            const float sc = valid ? s[j] * a.scale : -INFINITY;
            const float mt = warp_max(sc);
            const float m_new = fmaxf(m_run[j], mt);
            float p = 0.f, corr = 1.f;
            if (m_new != -INFINITY) {
                p = valid ? expf(sc - m_new) : 0.f;
                corr = expf(m_run[j] - m_new);  // 0 on the first contributing tile
            }
            l_run[j] = l_run[j] * corr + warp_sum(p);
            m_run[j] = m_new;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (i < npair) {
                    o[j][i][0] *= corr;
                    o[j][i][1] *= corr;
                }
            sm.p[(warp * 2 + j) * kAttnKeys + lane] = p;
        }
        __syncwarp();
        for (int jk = 0; jk < nt; ++jk) {
            const float p0 = sm.p[(warp * 2) * kAttnKeys + jk];
            const float p1 = sm.p[(warp * 2 + 1) * kAttnKeys + jk];
            const uint32_t* vr = reinterpret_cast<const uint32_t*>(sm.v[buf] + jk * hd);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                if (i < npair) {
                    const float2 v = kv_pair(vr[lane + 32 * i], a.kv_bf16);
                    o[0][i][0] += p0 * v.x;
                    o[0][i][1] += p0 * v.y;
                    o[1][i][0] += p1 * v.x;
                    o[1][i][1] += p1 * v.y;
                }
            }
        }
        __syncthreads();  // the buffer is refilled on the next trip
    }

    // Publish this split's partial result in shared memory (the query staging area).
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        float* op = sm.q + (warp * 2 + j) * hd;
#pragma unroll
        for (int i = 0; i < 8; ++i)
            if (i < npair) *reinterpret_cast<float2*>(op + 2 * lane + 64 * i) = make_float2(o[j][i][0], o[j][i][1]);
        if (lane == 0) sm.ml[warp * 2 + j] = make_float2(m_run[j], l_run[j]);
    }
    cluster.sync();

    // Combine across the cluster: CTA r owns rows 2r, 2r+1 of the chunk; one warp per
    // (row, 64-column group).
    const int ngroups = hd / 64;
    const int K = a.qh * hd;
    const BFragView bv = bfrag_view(bfrag, (K + 127) / 128 * 128, a.M);
    for (int w = warp; w < 2 * ngroups; w += kAttnThreads / 32) {
        const int r = split * 2 + w / ngroups, g = w % ngroups;
        const int qr = chunk * kAttnRows + r;
        if (qr >= R) continue;  // warp-uniform
        float mx = -INFINITY;
        for (int s = 0; s < kSplits; ++s) {
            const float2* rml = cluster.map_shared_rank(sm.ml, s);
            mx = fmaxf(mx, rml[r].x);
        }
        float n0 = 0.f, n1 = 0.f, den = 0.f;
        for (int s = 0; s < kSplits; ++s) {
            const float2 ml = cluster.map_shared_rank(sm.ml, s)[r];
            if (ml.y <= 0.f) continue;
            const float wgt = expf(ml.x - mx);
            const float2 op = *reinterpret_cast<const float2*>(cluster.map_shared_rank(sm.q, s) + r * hd + g * 64 + 2 * lane);
            n0 += wgt * op.x;
            n1 += wgt * op.y;
            den += wgt * ml.y;
        }
        const float inv = den > 0.f ? 1.0f / den : 0.f;
        const int m = qr / gqa, qhead = kvh_i * gqa + qr % gqa;
        bfrag_store_group(bv, a.M, m, (qhead * hd) / 64 + g, n0 * inv, n1 * inv, stage[warp]);
    }
    // A K that is not a multiple of 128 leaves one pad group per row: zero fragments.
    if ((K & 127) && blockIdx.y == 0 && blockIdx.z == 0 && split == 0)
        for (int m = warp; m < a.M; m += kAttnThreads / 32) bfrag_store_group(bv, a.M, m, K / 64, 0.f, 0.f, stage[warp]);
    cluster.sync();  // keep every CTA's shared memory alive until all remote reads are done
}

static size_t attn_smem_bytes(int hd) {
    return (size_t)kAttnRows * hd * 4 + 2 * ((size_t)kAttnKeys * (hd + 8) * 2 + (size_t)kAttnKeys * hd * 2) +
           kAttnRows * kAttnKeys * 4 + kAttnRows * sizeof(float2);
}

}  // namespace g4b

using namespace g4b;

cudaError_t g4b_attention(const AttnArgs& a, void* bfrag, cudaStream_t st, bool pdl) {
    if (a.hd % 64 || a.hd > 512 || a.qh % a.kvh) return cudaErrorInvalidValue;
    const int chunks = (a.M * (a.qh / a.kvh) + kAttnRows - 1) / kAttnRows;
    static bool attr_set = false;
    if (!attr_set) {
        cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)attn_smem_bytes(512));
        attr_set = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kSplits, a.kvh, chunks);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = attn_smem_bytes(a.hd);
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
    return cudaLaunchKernelEx(&cfg, attention_kernel, a, bfrag);
}
