// Multi-row GQA attention over the KV ring -- Attention.hlsl (shaders/Attention.hlsl:65-179)
// rebuilt so the KV cache is read ONCE per KV head for all M verify rows and all of that
// head's query heads (the reference dispatches one group per (row, query head), re-reading
// the cache M * q_heads/kv_heads times).
//
// Grid (kv head, row chunk of 16 query rows, key split). Each CTA streams 32-key tiles of K
// and V into shared memory, each warp owns two query rows, scores are fp32 dot products of
// the fp32 query with the rounded K, and an online softmax (running max / sum) accumulates
// the unnormalised output. Row m of the batch sits at position base+m and sees keys
// [max(0, base+m+1-window), base+m+1) (all keys from 0 on full-attention layers), which is
// the reference's per-row causal span (shaders/Attention.hlsl:82-86). Scale is a parameter
// (1.0 for Gemma 4, src/cpu_reference.cpp:508-510).
//
// A second kernel combines the key splits and writes the attention output directly as the
// o-projection's B fragments.
#include "bfrag.cuh"
#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"
#include "model_dev.h"

#include <algorithm>

namespace g4b {

constexpr int kAttnKeys = 32;    // keys per tile (one per lane)
constexpr int kAttnRows = 16;    // query rows per CTA (two per warp)
constexpr int kAttnThreads = 256;

__device__ __forceinline__ float2 kv_pair(uint32_t bits2, int bf16) {
    if (bf16) return make_float2(__uint_as_float(bits2 << 16), __uint_as_float(bits2 & 0xFFFF0000u));
    return __half22float2(*reinterpret_cast<const __half2*>(&bits2));
}

__global__ void __launch_bounds__(kAttnThreads) attention_kernel(AttnArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int hd = a.hd;
    const int kstride = hd + 8;  // halves; 16-byte pad keeps per-lane key rows conflict-free
    float* q_s = reinterpret_cast<float*>(smem_raw);                         // [16][hd]
    uint16_t* k_s = reinterpret_cast<uint16_t*>(q_s + kAttnRows * hd);      // [32][kstride]
    uint16_t* v_s = k_s + kAttnKeys * kstride;                              // [32][hd]
    float* p_s = reinterpret_cast<float*>(v_s + kAttnKeys * hd);            // [16][32]

    pdl_enter();
    const int kvh_i = blockIdx.x, chunk = blockIdx.y, split = blockIdx.z;
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
        q_s[i] = v;
    }

    // Key range of the whole batch, then this split's share.
    const int kmin = a.window ? max(0, base + 1 - a.window) : 0;
    const int kmax = base + a.M;
    const int per = (kmax - kmin + a.nsplit - 1) / a.nsplit;
    const int ks = kmin + split * per, ke = min(kmax, ks + per);

    // Two rows per warp.
    int row_m[2], row_head[2], row_lo[2], row_hi[2];
    bool row_ok[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const int qr = chunk * kAttnRows + warp * 2 + j;
        row_ok[j] = qr < R;
        row_m[j] = row_ok[j] ? qr / gqa : 0;
        row_head[j] = kvh_i * gqa + (row_ok[j] ? qr % gqa : 0);
        const int end = base + row_m[j] + 1;
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

    for (int t0 = ks; t0 < ke; t0 += kAttnKeys) {
        const int nt = min(kAttnKeys, ke - t0);
        __syncthreads();  // previous tile fully consumed (and q staged on the first trip)
        const int chunks_per_row = hd / 8;
        for (int i = threadIdx.x; i < kAttnKeys * chunks_per_row; i += kAttnThreads) {
            const int j = i / chunks_per_row, c8 = i % chunks_per_row;
            uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
            if (j < nt) {
                const size_t src = ((size_t)((t0 + j) % a.cap) * a.kvh + kvh_i) * hd + c8 * 8;
                kv = *reinterpret_cast<const uint4*>(a.k_ring + src);
                vv = *reinterpret_cast<const uint4*>(a.v_ring + src);
            }
            *reinterpret_cast<uint4*>(k_s + j * kstride + c8 * 8) = kv;
            *reinterpret_cast<uint4*>(v_s + j * hd + c8 * 8) = vv;
        }
        __syncthreads();

        // Scores: lane = key, two rows.
        float s[2] = {0.f, 0.f};
        const uint16_t* kr = k_s + lane * kstride;
        for (int d = 0; d < hd; d += 8) {
            const uint4 kb = *reinterpret_cast<const uint4*>(kr + d);
            const float2 k01 = kv_pair(kb.x, a.kv_bf16), k23 = kv_pair(kb.y, a.kv_bf16);
            const float2 k45 = kv_pair(kb.z, a.kv_bf16), k67 = kv_pair(kb.w, a.kv_bf16);
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const float4 qa = *reinterpret_cast<const float4*>(q_s + (warp * 2 + j) * hd + d);
                const float4 qb = *reinterpret_cast<const float4*>(q_s + (warp * 2 + j) * hd + d + 4);
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
            p_s[(warp * 2 + j) * kAttnKeys + lane] = p;
        }
        __syncwarp();
        for (int jk = 0; jk < nt; ++jk) {
            const float p0 = p_s[(warp * 2) * kAttnKeys + jk];
            const float p1 = p_s[(warp * 2 + 1) * kAttnKeys + jk];
            const uint32_t* vr = reinterpret_cast<const uint32_t*>(v_s + jk * hd);
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
        __syncwarp();
    }

    // Unnormalised partial output of this split.
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        if (!row_ok[j]) continue;
        const int row = row_m[j] * a.qh + row_head[j];
        float* op = a.o_part + ((size_t)split * a.M * a.qh + row) * hd;
#pragma unroll
        for (int i = 0; i < 8; ++i)
            if (i < npair) *reinterpret_cast<float2*>(op + 2 * lane + 64 * i) = make_float2(o[j][i][0], o[j][i][1]);
        if (lane == 0) a.ml_part[(size_t)split * a.M * a.qh + row] = make_float2(m_run[j], l_run[j]);
    }
}

// Combines key splits: out = sum_s e^(m_s - M) O_s / sum_s e^(m_s - M) l_s, one warp per
// (row, 64-column group) of the [M][qh*hd] output, written as B fragments.
__global__ void attn_combine_kernel(AttnArgs a, void* bfrag) {
    __shared__ __half stage[8][128];
    pdl_enter();
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int K = a.qh * a.hd;
    const int ng = K / 64;
    const BFragView v = bfrag_view(bfrag, (K + 127) / 128 * 128, a.M);
    for (int w = blockIdx.x * 8 + wib; w < a.M * ng; w += gridDim.x * 8) {
        const int m = w / ng, gi = w % ng;
        const int col = gi * 64 + 2 * lane;
        const int head = col / a.hd, d = col % a.hd;
        const int row = m * a.qh + head;
        float mx = -INFINITY;
        for (int s = 0; s < a.nsplit; ++s) mx = fmaxf(mx, a.ml_part[(size_t)s * a.M * a.qh + row].x);
        float num0 = 0.f, num1 = 0.f, den = 0.f;
        for (int s = 0; s < a.nsplit; ++s) {
            const float2 ml = a.ml_part[(size_t)s * a.M * a.qh + row];
            if (ml.y <= 0.f) continue;
            const float wgt = expf(ml.x - mx);
            const float2 op = *reinterpret_cast<const float2*>(a.o_part + ((size_t)s * a.M * a.qh + row) * a.hd + d);
            num0 += wgt * op.x;
            num1 += wgt * op.y;
            den += wgt * ml.y;
        }
        const float inv = den > 0.f ? 1.0f / den : 0.f;
        bfrag_store_group(v, a.M, m, gi, num0 * inv, num1 * inv, stage[wib]);
    }
    // Tail groups of a K that is not a multiple of 128 are zero fragments.
    const int Kp = (K + 127) / 128 * 128;
    for (int w = blockIdx.x * 8 + wib; w < a.M * (Kp - K) / 64; w += gridDim.x * 8) {
        const int m = w / ((Kp - K) / 64), gi = K / 64 + w % ((Kp - K) / 64);
        bfrag_store_group(v, a.M, m, gi, 0.f, 0.f, stage[wib]);
    }
}

static size_t attn_smem(int hd) {
    return (size_t)kAttnRows * hd * 4 + (size_t)kAttnKeys * (hd + 8) * 2 + (size_t)kAttnKeys * hd * 2 +
           kAttnRows * kAttnKeys * 4;
}

}  // namespace g4b

using namespace g4b;

int g4b_attn_nsplit(int kvh, int M, int qh, int hd) {
    (void)hd;
    const int chunks = (M * (qh / kvh) + kAttnRows - 1) / kAttnRows;
    const int want = 2 * 148;
    return std::max(1, std::min(64, want / std::max(1, kvh * chunks)));
}

cudaError_t g4b_attention(const AttnArgs& a, cudaStream_t st, bool pdl) {
    if (a.hd % 64 || a.hd > 512 || a.qh % a.kvh) return cudaErrorInvalidValue;
    const int chunks = (a.M * (a.qh / a.kvh) + kAttnRows - 1) / kAttnRows;
    const size_t sm = attn_smem(a.hd);
    static bool attr_set = false;
    if (!attr_set) {
        cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)attn_smem(512));
        attr_set = true;
    }
    return launch(attention_kernel, dim3(a.kvh, chunks, a.nsplit), dim3(kAttnThreads), sm, st, pdl, a);
}

cudaError_t g4b_attn_combine(const AttnArgs& a, void* bfrag, cudaStream_t st, bool pdl) {
    const int warps = a.M * ((a.qh * a.hd + 127) / 128 * 2);
    const int blocks = std::max(1, std::min(1184, (warps + 7) / 8));
    return launch(attn_combine_kernel, dim3(blocks), dim3(256), 0, st, pdl, a, bfrag);
}
