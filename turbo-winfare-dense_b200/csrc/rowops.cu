// Row-wise kernels around the verify GEMM. Each consumes a GEMM's split-K slots (or an
// all-reduced matrix), applies the layer's elementwise/normalisation step in fp32 in the
// order src/cpu_reference.cpp uses, and produces the next GEMM's B fragments, so no
// activation is ever converted twice:
//   embed_norm   token gather x sqrt(d) (src/cpu_reference.cpp:260-291) + input RMSNorm
//   qkv_epi      q/k RMSNorm*w + NeoX RoPE, v unweighted RMSNorm (raw k on layers without
//                v_proj), K/V rounded and written to the ring (:398-498, QKVEpilogue.hlsl,
//                KVWrite.hlsl) -- one CTA per (row, head), one thread per rotary pair
//   rowepi       post-attention: h += rmsnorm(o)*w_post_attn; x = rmsnorm(h)*w_pre_ffn
//                (:560-567); post-FFN: h = (h + rmsnorm(down)*w_post_ffn) * layer_scalar,
//                then the next layer's input norm or the final norm (:583-629). One CTA
//                (narrow rows) or one 12-CTA cluster (wide rows, DSMEM reduction) per row:
//                slot sums and statistics, the two RMS factors, then every column.
//   geglu        gelu_tanh(gate) * up (:568-581, GeGLU.hlsl)
#include <cooperative_groups.h>

#include "bfrag.cuh"
#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"
#include "model_dev.h"
#include "rowmath.cuh"
#include "tma.cuh"

#include <algorithm>

namespace cg = cooperative_groups;

namespace g4b {

// Writes a full row x[0..K) (in shared memory) as GEMM operands, one warp per 64-group: B
// fragments for a verify batch, the wide layout (with the row's scale) for a prefill chunk.
// Block-collective; `red` is 32 floats of shared scratch.
__device__ __forceinline__ void row_to_bfrags(const float* xs, int K, int M, int m, void* bfrag, __half* stage,
                                              float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int Kp = (K + 127) / 128 * 128;
    const BFragView v = bfrag_view(bfrag, Kp, M);
    float inv_e = 1.f;
    if (M > kMaxM) {
        float amax = 0.f;
        for (int c = threadIdx.x; c < K; c += blockDim.x) amax = fmaxf(amax, fabsf(xs[c]));
        const float E = wide_row_scale(block_max(amax, red));
        inv_e = 1.0f / E;
        if (threadIdx.x == 0) v.erow[m] = E;
    }
    for (int gi = warp; gi < Kp / 64; gi += nw) {
        const int k = gi * 64 + 2 * lane;
        const float x0 = k < K ? xs[k] : 0.f, x1 = k + 1 < K ? xs[k + 1] : 0.f;
        if (M > kMaxM) wide_store_group(v, m, gi, x0, x1, inv_e);
        else bfrag_store_group(v, M, m, gi, x0, x1, stage + warp * 128);
    }
}

// ---------------------------------------------------------------- embedding + input norm

__global__ void embed_norm_kernel(const StepParams* __restrict__ sp, const uint32_t* __restrict__ ew,
                                  const uint16_t* __restrict__ es, const uint16_t* __restrict__ eb, int V, int d,
                                  const uint16_t* __restrict__ w_in, float* __restrict__ h_out, void* bfrag, int M) {
    extern __shared__ float smem[];
    float* xs = smem;                                   // [d]
    __half* stage = reinterpret_cast<__half*>(xs + d);  // [warps][128]
    __shared__ float red[32];
    pdl_enter();
    const int m = blockIdx.x;
    const uint32_t tok = sp->tokens[m] % (uint32_t)V;
    const float scale = sqrtf((float)d);
    const uint32_t* wr = ew + (size_t)tok * (d / 8);
    const uint16_t* sr = es + (size_t)tok * (d / 64);
    const uint16_t* br = eb + (size_t)tok * (d / 64);
    float ss = 0.f;
    for (int c = threadIdx.x; c < d; c += blockDim.x) {
        const uint32_t q = (wr[c >> 3] >> ((c & 7) * 4)) & 0xFu;
        const float v = ((float)q * bf16_to_f32(sr[c >> 6]) + bf16_to_f32(br[c >> 6])) * scale;
        h_out[(size_t)m * d + c] = v;
        xs[c] = v;
        ss += v * v;
    }
    const float r = inv_rms(block_sum(ss, red), d);
    for (int c = threadIdx.x; c < d; c += blockDim.x) xs[c] = xs[c] * r * bf16_to_f32(w_in[c]);
    __syncthreads();
    row_to_bfrags(xs, d, M, m, bfrag, stage, red);
}

// ---------------------------------------------------------------- MTP drafter input

// MtpRunner's step input (src/mtp_runner.cpp:318-327): x = [e(t) * sqrt(bb); h] as the
// pre-projection's B fragments (one row, K = 2 * bb). e(t) is the target's dequantised embedding
// row of sp->tokens[0] (ForwardRunner::get_token_embedding, src/runner.cpp:2359-2380); h is row
// sp->aux of the target's final normed hidden states on a round's first step, else the previous
// step's post-projection (its split-K slots).
__global__ void mtp_input_kernel(const StepParams* __restrict__ sp, const uint32_t* __restrict__ ew,
                                 const uint16_t* __restrict__ es, const uint16_t* __restrict__ eb, int V, int bb,
                                 const float* __restrict__ hidden, GemmOut post, void* bfrag) {
    extern __shared__ float smem[];
    float* xs = smem;                                        // [2 * bb]
    __half* stage = reinterpret_cast<__half*>(xs + 2 * bb);  // [warps][128]
    __shared__ float red[32];
    pdl_enter();
    const uint32_t tok = sp->tokens[0] % (uint32_t)V;
    const float scale = sqrtf((float)bb);
    const uint32_t* wr = ew + (size_t)tok * (bb / 8);
    const uint16_t* sr = es + (size_t)tok * (bb / 64);
    const uint16_t* br = eb + (size_t)tok * (bb / 64);
    for (int c = threadIdx.x; c < bb; c += blockDim.x) {
        const uint32_t q = (wr[c >> 3] >> ((c & 7) * 4)) & 0xFu;
        xs[c] = ((float)q * bf16_to_f32(sr[c >> 6]) + bf16_to_f32(br[c >> 6])) * scale;
    }
    if (hidden) {
        const float* hr = hidden + (size_t)sp->aux * bb;
        for (int c = threadIdx.x; c < bb; c += blockDim.x) xs[bb + c] = hr[c];
    } else {
        for (int c = 2 * threadIdx.x; c < bb; c += 2 * blockDim.x) {
            const float2 v = gemm_out_pair(post, 0, c);
            xs[bb + c] = v.x;
            xs[bb + c + 1] = v.y;
        }
    }
    __syncthreads();
    row_to_bfrags(xs, 2 * bb, 1, 0, bfrag, stage, red);
}

// ---------------------------------------------------------------- Q/K/V epilogue

// One CTA per (row m, head): heads [0, qh) are query heads, [qh, qh + kvh) KV heads. Thread i
// (blockDim = hd/2) holds the NeoX pair (i, i + hd/2) -- its two elements and their rotation
// stay in registers, every slot load of the pair is in flight together, and the per-head RMS
// is a block reduction. Restates the reference's q/k/v norms, RoPE and FP16 cache rounding
// (src/cpu_reference.cpp:452-498).

// Elements r0 + i and r0 + i + half of row m (DENSE: the GEMM wrote a dense matrix).
template <bool DENSE>
__device__ __forceinline__ float2 load_pair(const GemmOut& o, int m, int r0, int half) {
    const int i = threadIdx.x;
    if (DENSE) {
        const float* src = o.y + (size_t)m * o.ld + r0 + i;
        return make_float2(src[0], src[half]);
    }
    const int ra = r0 + i, rb = r0 + i + half;
    const float* pj[2] = {slot_base(o.part, m, ra >> 8) + (ra & 255), slot_base(o.part, m, rb >> 8) + (rb & 255)};
    const int nsa = slot_count(o.part, ra >> 8);
    const int nsb = (rb >> 8) == (ra >> 8) ? nsa : slot_count(o.part, rb >> 8);
    const int nsj[2] = {nsa, nsb};
    float v[2];
    slot_sums_each<2, 16>(pj, nsj, max(nsa, nsb), v);
    return make_float2(v[0], v[1]);
}

// DENSE (a prefill chunk's dense GEMM output) is a separate instance: the slot sums' registers
// would otherwise cut the CTAs resident per SM for the thousands of CTAs of a 128-row chunk.
template <bool DENSE>
__global__ void __launch_bounds__(256, 3) qkv_epi_kernel(QkvEpiArgs a) {
    __shared__ float2 red2[32];
    pdl_launch_dependents();
    const int heads = a.qh + a.kvh;
    const int m = blockIdx.x / heads, head = blockIdx.x % heads;
    const int hd = a.hd, half = hd / 2, i = threadIdx.x;
    const int nq = a.qh * hd, nk = a.kvh * hd;
    const bool is_q = head < a.qh;
    const int kvh = head - a.qh;
    // Before waiting on the GEMM: the norm weights and the rotation, which depend only on the
    // position (base_pos is written by a pass's last kernel alone, and every pass starts with a
    // kernel launched without programmatic overlap, so it is stable here).
    const int pos = a.sp->base_pos + m + a.pos_offset;
    const uint16_t* wn = is_q ? a.q_norm : a.k_norm;
    const float wa = bf16_to_f32(wn[i]), wb = bf16_to_f32(wn[i + half]);
    float rc = 1.f, rs = 0.f;
    if (i < a.rotated) {
        const float freq = 1.0f / powf(a.theta, (float)(2 * i) / (float)hd);
        const float ang = (float)pos * freq;
        rc = cosf(ang);
        rs = sinf(ang);
    }
    pdl_wait();
    // A KV head's k and v rows load together and their two sums of squares share one
    // reduction (V: unweighted norm of v_proj, or of the RAW k on layers without v_proj).
    float2 x = load_pair<DENSE>(a.qkv, m, is_q ? head * hd : nq + kvh * hd, half);
    const float2 v = !is_q && a.has_v ? load_pair<DENSE>(a.qkv, m, nq + nk + kvh * hd, half) : x;
    const float2 ss = block_sum2(make_float2(x.x * x.x + x.y * x.y, v.x * v.x + v.y * v.y), red2);
    const float r = inv_rms(ss.x, hd);
    if (!is_q) {
        const float rv = inv_rms(ss.y, hd);
        uint16_t* vd = a.v_ring + ((size_t)(pos % a.cap) * a.kvh + kvh) * hd;
        const float t0 = v.x * rv, t1 = v.y * rv;
        vd[i] = a.kv_bf16 ? bf16_bits_rne(t0) : f16_bits_like_reference(t0);
        vd[i + half] = a.kv_bf16 ? bf16_bits_rne(t1) : f16_bits_like_reference(t1);
    }
    x.x = x.x * r * wa;
    x.y = x.y * r * wb;
    // NeoX rotary on the first `rotated` pairs.
    if (i < a.rotated) {
        const float x0 = x.x, x1 = x.y;
        x.x = x0 * rc - x1 * rs;
        x.y = x0 * rs + x1 * rc;
    }
    if (is_q) {
        float* qd = a.q_out + ((size_t)m * a.qh + head) * hd;
        qd[i] = x.x;
        qd[i + half] = x.y;
    } else {
        uint16_t* kd = a.k_ring + ((size_t)(pos % a.cap) * a.kvh + kvh) * hd;
        kd[i] = a.kv_bf16 ? bf16_bits_rne(x.x) : f16_bits_like_reference(x.x);
        kd[i + half] = a.kv_bf16 ? bf16_bits_rne(x.y) : f16_bits_like_reference(x.y);
    }
}

// ---------------------------------------------------------------- norm/residual epilogues

// Narrow rows (d <= 1024, and prefill rows up to d = 6144): one CTA per row, the statistics
// reduced in the CTA. Wider verify rows: one 12-CTA cluster per row; CTA r owns groups
// [r*gpc, (r+1)*gpc) (gpc = ceil(groups / 12)), each warp up to kEpiGroupsPerWarp of them, and
// the cluster adds the CTA sums in rank order through distributed shared memory, so every CTA
// derives the same two RMS factors. In both forms a warp holds its columns in registers from
// start to finish: phase 1 sums the split-K slots and the sums of y^2, h^2, h*c and c^2
// (c = y * w1); phase 2 finishes the columns.
// 12 CTAs: measured against 8 and 16 on the 31B verify pass and the E2B drafter step (both
// about 0.6 % faster than with 16); a non-portable size, which B200 allows up to 16.
constexpr int kEpiClusters = 12;
constexpr int kEpiWarps = 8;         // warps per CTA in the cluster form
constexpr int kEpiGroupsPerWarp = 2;  // d <= 12 CTAs x 8 warps x 2 groups x 64 = 12288
constexpr int kEpiMaxWarps = 32;

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Tensor parallelism: publish this rank's flag (its partial is complete once this kernel
// runs) and wait, bounded, for every peer's.
__device__ void tp_sync(const TpGather& tg, bool publisher) {
    if (threadIdx.x == 0) {
        const unsigned epoch = *tg.seq * 256u + (unsigned)tg.step + 1u;
        if (publisher) {
            __threadfence_system();
            asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(tg.own_flag), "r"(epoch) : "memory");
        }
        for (int r = 0; r < tg.n; ++r) {
            if (r == tg.rank) continue;
            const uint64_t t0 = global_ns();
            while ((int)(ld_acquire_sys(tg.flag[r]) - epoch) < 0) {
                if (global_ns() - t0 > kWaitLimitNs) {
                    atomicExch(tg.err, 3);
                    break;
                }
            }
        }
    }
    __syncthreads();
}

// Tensor parallelism, verify rows: values travel with their step's epoch in the same 8-byte word
// ({value bits, epoch}), written by one 16-byte store per column pair, so a reader that sees both
// epochs of a pair sees both values; no fence or separate flag is needed. Stores and polls are
// volatile (relaxed, system scope) and bypass L1.
__device__ __forceinline__ void st_volatile_v4(void* p, uint4 v) {
    asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}
__device__ __forceinline__ uint4 ld_volatile_v4(const void* p) {
    uint4 v;
    asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}
// Columns c, c+1 of row m from every rank, added in rank order (this rank's own from `mine`).
// Waits, bounded, for each peer's words of this step.
__device__ float2 tp_ll_sum(const TpGather& tg, int m, int d, int c, float2 mine, unsigned epoch) {
    float2 s = make_float2(0.f, 0.f);
    for (int r = 0; r < tg.n; ++r) {
        float2 v = mine;
        if (r != tg.rank) {
            const uint2* src = tg.recv + ((size_t)r * kMaxM + m) * d + c;
            uint4 w = ld_volatile_v4(src);
            if (w.y != epoch || w.w != epoch) {
                const uint64_t t0 = global_ns();
                do {
                    w = ld_volatile_v4(src);
                    if (global_ns() - t0 > kWaitLimitNs) {
                        atomicExch(tg.err, 3);
                        break;
                    }
                } while (w.y != epoch || w.w != epoch);
            }
            v = make_float2(__uint_as_float(w.x), __uint_as_float(w.z));
        }
        s.x += v.x;
        s.y += v.y;
    }
    return s;
}

// Columns c, c+1 of row m summed over the ranks in rank order (peer partials bypass the caches).
__device__ __forceinline__ float2 tp_pair(const TpGather& tg, int m, int ld, int c) {
    float2 s = make_float2(0.f, 0.f);
    for (int r = 0; r < tg.n; ++r) {
        const float2* p = reinterpret_cast<const float2*>(tg.y[r] + (size_t)m * ld + c);
        const float2 v = r == tg.rank ? __ldcg(p) : __ldcv(p);
        s.x += v.x;
        s.y += v.y;
    }
    return s;
}

template <bool CLUSTER, int GPW = kEpiGroupsPerWarp>
__global__ void __launch_bounds__(CLUSTER ? kEpiWarps * 32 : kEpiMaxWarps * 32) rowepi_kernel(GemmOut o, TpGather tg,
                                                                    const float* __restrict__ h_in,
                                                                    float* __restrict__ h_out,
                                                                    const uint16_t* __restrict__ w1, float out_scale,
                                                                    const uint16_t* __restrict__ w2, int d,
                                                                    void* bfrag, int M, int frag_row0,
                                                                    float* __restrict__ x_out) {
    __shared__ float4 red[kEpiMaxWarps];
    __shared__ float red_max[32];
    __shared__ float4 cta_sum;
    __shared__ __half stage[kEpiMaxWarps][128];
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int rank = CLUSTER ? (int)cg::this_cluster().block_rank() : 0;
    const int m = blockIdx.y;
    const int Kp = (d + 127) / 128 * 128;
    const int ngp = Kp / 64;
    const int gpc = CLUSTER ? (ngp + kEpiClusters - 1) / kEpiClusters : ngp;
    const int g_end = min(ngp, (rank + 1) * gpc);
    // The two norm weights of this thread's columns do not depend on the producer: load them
    // before the wait (in the 1024-thread form, with its 64 registers, after it).
    float2 wv1[GPW], wv2[GPW];
    auto load_w = [&] {
#pragma unroll
        for (int j = 0; j < GPW; ++j) {
            const int c0 = (rank * gpc + warp + nw * j) * 64 + 2 * lane;
            wv1[j] = wv2[j] = make_float2(0.f, 0.f);
            if (rank * gpc + warp + nw * j < g_end && c0 < d) {
                wv1[j] = w1 ? make_float2(bf16_to_f32(w1[c0]), bf16_to_f32(w1[c0 + 1])) : make_float2(1.f, 1.f);
                wv2[j] = make_float2(bf16_to_f32(w2[c0]), bf16_to_f32(w2[c0 + 1]));
            }
        }
    };
    constexpr bool kPreloadW = CLUSTER || GPW <= 2;
    if constexpr (kPreloadW) load_w();
    pdl_wait();
    // Weight of column c (= (rank * gpc + warp + nw * j) * 64 + 2 * lane + e).
    auto wt1 = [&](int j, int e, int c) {
        return kPreloadW ? (e ? wv1[j].y : wv1[j].x) : (w1 ? bf16_to_f32(w1[c]) : 1.f);
    };
    auto wt2 = [&](int j, int e, int c) { return kPreloadW ? (e ? wv2[j].y : wv2[j].x) : bf16_to_f32(w2[c]); };
    // Under tensor parallelism with split-K slots (verify rows): this rank's sums of the CTA's
    // columns go to every rank's receive area; the ranks' sums are then added in rank order from
    // local memory. A dense GEMM output (prefill chunks) is read from the ranks' buffers instead.
    const bool tp_push = tg.n > 1 && o.part.part != nullptr;
    float2 mine[GPW];
    unsigned epoch = 0;
    if (tg.n > 1) {
        if (tp_push) {
            epoch = *tg.seq * 256u + (unsigned)tg.step + 1u;
#pragma unroll
            for (int j = 0; j < GPW; ++j) {
                const int gi = rank * gpc + warp + nw * j;
                const int c0 = gi * 64 + 2 * lane;
                mine[j] = make_float2(0.f, 0.f);
                if (gi < g_end && c0 < d) {
                    mine[j] = gemm_out_pair(o, m, c0);
                    const uint4 w = make_uint4(__float_as_uint(mine[j].x), epoch, __float_as_uint(mine[j].y), epoch);
                    for (int r = 0; r < tg.n; ++r)
                        if (r != tg.rank) st_volatile_v4(tg.push_dst[r] + (size_t)m * d + c0, w);
                }
            }
        } else {
            tp_sync(tg, blockIdx.x == 0 && blockIdx.y == 0);  // the GEMM wrote the buffer itself
        }
    }

    float2 y[GPW], h[GPW];
    // A cluster CTA with at least twice as many warps as groups (d = 1536: 2 groups, 8 warps)
    // spreads each group's split-K slots over wpg warps, so a long slot list (a down projection
    // split 48 ways) costs one round of loads instead of several. Warp w sums share w / gpc of
    // group w % gpc's slots; warp g < gpc then adds the shares in share order.
    const int wpg = (CLUSTER && o.part.part && tg.n == 1) ? nw / gpc : 1;  // block-uniform
    if (wpg >= 2) {
        __shared__ float2 share_sum[kEpiWarps][32];
        const int gl = warp % gpc, share = warp / gpc;
        const int c0 = (rank * gpc + gl) * 64 + 2 * lane;
        float2 ps = make_float2(0.f, 0.f);
        if (share < wpg && rank * gpc + gl < g_end && c0 < d) {
            const int ns = slot_count(o.part, c0 >> 8);
            ps = slot_pair_range(o.part, m, c0, ns * share / wpg, ns * (share + 1) / wpg);
        }
        share_sum[warp][lane] = ps;
        __syncthreads();
        if (warp < gpc) {
            y[0] = share_sum[warp][lane];
            for (int s = 1; s < wpg; ++s) {
                y[0].x += share_sum[warp + s * gpc][lane].x;
                y[0].y += share_sum[warp + s * gpc][lane].y;
            }
        }
    }
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int j = 0; j < GPW; ++j) {
        const int gi = rank * gpc + warp + nw * j;
        const int c0 = gi * 64 + 2 * lane;
        if (wpg < 2 || j > 0 || warp >= gpc) y[j] = make_float2(0.f, 0.f);
        h[j] = make_float2(0.f, 0.f);
        if (gi < g_end && c0 < d) {
            if (wpg < 2) {
                if (tp_push) {
                    y[j] = tp_ll_sum(tg, m, d, c0, mine[j], epoch);
                } else {
                    y[j] = tg.n > 1 ? tp_pair(tg, m, d, c0) : gemm_out_pair(o, m, c0);
                }
            }
            if (h_in) h[j] = *reinterpret_cast<const float2*>(h_in + (size_t)m * d + c0);
            const float ca = y[j].x * wt1(j, 0, c0), cb = y[j].y * wt1(j, 1, c0 + 1);
            acc.x += y[j].x * y[j].x + y[j].y * y[j].y;
            acc.y += h[j].x * h[j].x + h[j].y * h[j].y;
            acc.z += h[j].x * ca + h[j].y * cb;
            acc.w += ca * ca + cb * cb;
        }
    }
    acc.x = warp_sum(acc.x);
    acc.y = warp_sum(acc.y);
    acc.z = warp_sum(acc.z);
    acc.w = warp_sum(acc.w);
    if (lane == 0) red[warp] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        float4 t = red[0];
        for (int i = 1; i < nw; ++i) {
            t.x += red[i].x; t.y += red[i].y; t.z += red[i].z; t.w += red[i].w;
        }
        cta_sum = t;
    }
    float4 t;
    if constexpr (CLUSTER) {
        cg::cluster_group cluster = cg::this_cluster();
        cluster.sync();
        float4 u[kEpiClusters];
#pragma unroll
        for (int r = 0; r < kEpiClusters; ++r) u[r] = *cluster.map_shared_rank(&cta_sum, r);  // all in flight
        t = u[0];
#pragma unroll
        for (int r = 1; r < kEpiClusters; ++r) {
            t.x += u[r].x; t.y += u[r].y; t.z += u[r].z; t.w += u[r].w;
        }
        // Every CTA must have read the others' sums before any of them exits: arrive once the
        // sums are in registers (the operands tie the arrival to the loads' completion), wait
        // at the end, so the barrier's latency overlaps the column work below.
        asm volatile("barrier.cluster.arrive.release.aligned;" ::"f"(t.x), "f"(t.y), "f"(t.z), "f"(t.w) : "memory");
    } else {
        __syncthreads();
        t = cta_sum;
    }
    const float r1 = w1 ? inv_rms(t.x, d) : 1.f;  // plain mode: y enters the residual unnormalised
    const float s2 = out_scale * out_scale * (t.y + 2.0f * r1 * t.z + r1 * r1 * t.w);
    const float r2 = inv_rms(fmaxf(s2, 0.f), d);
    // Fragments for rows frag_row0.. only, as rows 0.. of an (M - frag_row0)-row batch (a
    // prefill chunk's final norm feeds the LM head its last row alone).
    const int Mf = M - frag_row0, mf = m - frag_row0;
    const BFragView bv = bfrag_view(bfrag, Kp, Mf);
    float xv[GPW][2];
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < GPW; ++j) {
        const int gi = rank * gpc + warp + nw * j;
        xv[j][0] = xv[j][1] = 0.f;
        if (gi >= g_end) continue;  // warp-uniform
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int c = gi * 64 + 2 * lane + e;
            if (c < d) {
                const float yy = e ? y[j].y : y[j].x, hh = e ? h[j].y : h[j].x;
                const float a = __fmul_rn(__fmul_rn(yy, r1), wt1(j, e, c));
                const float hn = __fmul_rn(__fadd_rn(hh, a), out_scale);
                h_out[(size_t)m * d + c] = hn;
                xv[j][e] = __fmul_rn(__fmul_rn(hn, r2), wt2(j, e, c));
                if (x_out && mf >= 0) x_out[(size_t)mf * d + c] = xv[j][e];
                amax = fmaxf(amax, fabsf(xv[j][e]));
            }
        }
    }
    float inv_e = 1.f;
    if (Mf > kMaxM) {  // wide layout (one CTA holds the whole row): the row's scale first
        const float E = wide_row_scale(block_max(amax, red_max));
        inv_e = 1.0f / E;
        if (threadIdx.x == 0) bv.erow[mf] = E;
    }
#pragma unroll
    for (int j = 0; j < GPW; ++j) {
        const int gi = rank * gpc + warp + nw * j;
        if (gi >= g_end || mf < 0) continue;  // warp-uniform / block-uniform
        if (Mf > kMaxM) wide_store_group(bv, mf, gi, xv[j][0], xv[j][1], inv_e);
        else bfrag_store_group(bv, Mf, mf, gi, xv[j][0], xv[j][1], stage[warp]);
    }
    if constexpr (CLUSTER) asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// ---------------------------------------------------------------- GeGLU

// One warp per (row, 64-group) of the F-wide activation; gate rows [0, F), up rows [F, 2F).
__global__ void geglu_kernel(GemmOut gu, int F, void* bfrag, int M) {
    __shared__ __half stage[8][128];
    pdl_enter();
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int Fp = (F + 127) / 128 * 128;
    const int ng = Fp / 64;
    const BFragView v = bfrag_view(bfrag, Fp, M);
    for (int w = blockIdx.x * 8 + wib; w < M * ng; w += gridDim.x * 8) {
        const int m = w / ng, gi = w % ng;
        const int k = gi * 64 + 2 * lane;
        float x0 = 0.f, x1 = 0.f;
        if (k < F) {
            float2 g, u;
            gemm_out_two_pairs(gu, m, k, F + k, g, u);
            x0 = gelu_tanh_dev(g.x) * u.x;
            x1 = gelu_tanh_dev(g.y) * u.y;
        }
        bfrag_store_group(v, M, m, gi, x0, x1, stage[wib]);
    }
}

// Prefill rows: one CTA per row, so the row's scale is known before the wide-layout stores.
// Pass 1 finds max |gelu(g) u| over the row; pass 2 recomputes and stores (the inputs are in L2).
__global__ void __launch_bounds__(1024) geglu_wide_kernel(GemmOut gu, int F, void* bfrag, int M) {
    __shared__ float red[32];
    pdl_enter();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int m = blockIdx.x;
    const int Fp = (F + 127) / 128 * 128;
    const int ng = Fp / 64;
    const BFragView v = bfrag_view(bfrag, Fp, M);
    const float* yr = gu.y + (size_t)m * gu.ld;  // a prefill GEMM's dense output
    auto value = [&](int k, float2& x) {
        x = make_float2(0.f, 0.f);
        if (k < F) {
            const float2 g = *reinterpret_cast<const float2*>(yr + k), u = *reinterpret_cast<const float2*>(yr + F + k);
            x.x = gelu_tanh_dev(g.x) * u.x;
            x.y = gelu_tanh_dev(g.y) * u.y;
        }
    };
    float amax = 0.f;
    for (int gi = warp; gi < ng; gi += nw) {
        float2 x;
        value(gi * 64 + 2 * lane, x);
        amax = fmaxf(amax, fmaxf(fabsf(x.x), fabsf(x.y)));
    }
    const float E = wide_row_scale(block_max(amax, red));
    if (threadIdx.x == 0) v.erow[m] = E;
    const float inv_e = 1.0f / E;
    for (int gi = warp; gi < ng; gi += nw) {
        float2 x;
        value(gi * 64 + 2 * lane, x);
        wide_store_group(v, m, gi, x.x, x.y, inv_e);
    }
}

// ---------------------------------------------------------------- plain conversion

// x [M][ldx] fp32 -> wide layout for 17..128 rows: one CTA per row (its scale first).
__global__ void __launch_bounds__(1024) wide_from_f32_kernel(const float* __restrict__ x, int ldx, int M, int K,
                                                             void* bfrag) {
    __shared__ float red[32];
    pdl_enter();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int m = blockIdx.x;
    const int Kp = (K + 127) / 128 * 128;
    const BFragView v = bfrag_view(bfrag, Kp, M);
    const float* xr = x + (size_t)m * ldx;
    float amax = 0.f;
    for (int c = threadIdx.x; c < K; c += blockDim.x) amax = fmaxf(amax, fabsf(xr[c]));
    const float E = wide_row_scale(block_max(amax, red));
    if (threadIdx.x == 0) v.erow[m] = E;
    const float inv_e = 1.0f / E;
    for (int gi = warp; gi < Kp / 64; gi += nw) {
        const int k = gi * 64 + 2 * lane;
        wide_store_group(v, m, gi, k < K ? xr[k] : 0.f, k + 1 < K ? xr[k + 1] : 0.f, inv_e);
    }
}

// x [M][ldx] fp32 -> B fragments. One warp per (row, 64-group); groups past K are zeros.
__global__ void bfrag_from_f32_kernel(const float* __restrict__ x, int ldx, int M, int K, void* bfrag) {
    __shared__ __half stage[8][128];
    pdl_enter();
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int Kp = (K + 127) / 128 * 128;
    const int ngroups = Kp / 64;
    const BFragView v = bfrag_view(bfrag, Kp, M);
    const int total = M * ngroups;
    for (int w = blockIdx.x * 8 + wib; w < total; w += gridDim.x * 8) {
        const int m = w / ngroups, gi = w % ngroups;
        const int k = gi * 64 + 2 * lane;
        const float x0 = k < K ? x[(size_t)m * ldx + k] : 0.f;
        const float x1 = k + 1 < K ? x[(size_t)m * ldx + k + 1] : 0.f;
        bfrag_store_group(v, M, m, gi, x0, x1, stage[wib]);
    }
}

}  // namespace g4b

using namespace g4b;

static int grid_for_warps(int warps) { return std::max(1, std::min(1184, (warps + 7) / 8)); }

cudaError_t g4b_bfrag_from_f32(const float* x, int ldx, int M, int K, void* bfrag, cudaStream_t st, bool pdl) {
    if (M > kMaxM) return launch(wide_from_f32_kernel, dim3(M), dim3(1024), 0, st, pdl, x, ldx, M, K, bfrag);
    const int ngroups = (K + 127) / 128 * 2;
    return launch(bfrag_from_f32_kernel, dim3(grid_for_warps(M * ngroups)), dim3(256), 0, st, pdl, x, ldx, M, K,
                  bfrag);
}

static size_t row_smem(int d, int threads) { return (size_t)d * sizeof(float) + (threads / 32) * 128 * sizeof(__half); }

cudaError_t g4b_embed_norm(const StepParams* sp, const uint32_t* ew, const uint16_t* es, const uint16_t* eb, int V,
                           int d, const uint16_t* w_in, float* h_out, void* bfrag, int M, cudaStream_t st, bool pdl) {
    const int th = 512;
    return launch(embed_norm_kernel, dim3(M), dim3(th), row_smem(d, th), st, pdl, sp, ew, es, eb, V, d, w_in, h_out,
                  bfrag, M);
}

cudaError_t g4b_mtp_input(const StepParams* sp, const uint32_t* ew, const uint16_t* es, const uint16_t* eb, int V,
                          int bb, const float* hidden, const GemmOut& post, void* bfrag, cudaStream_t st, bool pdl) {
    if (bb % 64) return cudaErrorInvalidValue;
    const int th = 512;
    const size_t smem = row_smem(2 * bb, th);
    static bool attr_set = false;
    if (!attr_set) {
        const cudaError_t e =
            cudaFuncSetAttribute(mtp_input_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    if (smem > 96 * 1024) return cudaErrorInvalidValue;
    return launch(mtp_input_kernel, dim3(1), dim3(th), smem, st, pdl, sp, ew, es, eb, V, bb, hidden, post, bfrag);
}

cudaError_t g4b_qkv_epi(const QkvEpiArgs& a, cudaStream_t st, bool pdl) {
    if (a.hd % 64 || a.hd > 1024 || a.rotated > a.hd / 2) return cudaErrorInvalidValue;
    if (!a.qkv.part.part)
        return launch(qkv_epi_kernel<true>, dim3(a.M * (a.qh + a.kvh)), dim3(a.hd / 2), 0, st, pdl, a);
    return launch(qkv_epi_kernel<false>, dim3(a.M * (a.qh + a.kvh)), dim3(a.hd / 2), 0, st, pdl, a);
}

cudaError_t g4b_rowepi(const GemmOut& o, const TpGather& tg, const float* h_in, float* h_out, const uint16_t* w1,
                       float out_scale, const uint16_t* w2, int d, void* bfrag, int M, cudaStream_t st, bool pdl,
                       int frag_row0, float* x_out) {
    if ((o.ld | d) & 1) return cudaErrorInvalidValue;  // float2 loads
    if (frag_row0 < 0 || frag_row0 >= M) return cudaErrorInvalidValue;
    if (tg.n < 1 || tg.n > kMaxTp) return cudaErrorInvalidValue;
    const int ngp = (d + 127) / 128 * 2;
    // Rows of up to 16 groups (d <= 1024): one CTA per row, one warp per group. Wider verify
    // rows spread their slot sums over a 12-CTA cluster (measured faster from d = 1536 up).
    if (ngp <= 16)
        return launch(rowepi_kernel<false>, dim3(1, M), dim3(ngp * 32), 0, st, pdl, o, tg, h_in, h_out, w1, out_scale,
                      w2, d, bfrag, M, frag_row0, x_out);
    // A prefill chunk has rows enough to fill the GPU: one CTA per row (each warp up to three
    // groups) instead of a 12-CTA cluster per row.
    if (M > kMaxM && ngp <= kEpiMaxWarps)
        return launch(rowepi_kernel<false>, dim3(1, M), dim3(ngp * 32), 0, st, pdl, o, tg, h_in, h_out, w1, out_scale,
                      w2, d, bfrag, M, frag_row0, x_out);
    if (M > kMaxM && ngp <= 3 * kEpiMaxWarps)
        return launch(rowepi_kernel<false, 3>, dim3(1, M), dim3(kEpiMaxWarps * 32), 0, st, pdl, o, tg, h_in, h_out, w1,
                      out_scale, w2, d, bfrag, M, frag_row0, x_out);
    // Beyond here the cluster form: a prefill chunk's wide layout needs the row in one CTA.
    if (M - frag_row0 > kMaxM) return cudaErrorInvalidValue;
    if ((ngp + kEpiClusters - 1) / kEpiClusters > kEpiWarps * kEpiGroupsPerWarp) return cudaErrorInvalidValue;
    static bool attr_set = false;
    if (!attr_set) {
        const cudaError_t e =
            cudaFuncSetAttribute(rowepi_kernel<true>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kEpiClusters, M);
    cfg.blockDim = dim3(kEpiWarps * 32);
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kEpiClusters;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, rowepi_kernel<true>, o, tg, h_in, h_out, w1, out_scale, w2, d, bfrag, M, frag_row0, x_out);
}

cudaError_t g4b_geglu(const GemmOut& gu, int F, void* bfrag, int M, cudaStream_t st, bool pdl) {
    if ((gu.ld | F) & 1) return cudaErrorInvalidValue;  // float2 loads
    if (M > kMaxM) {  // prefill: the GEMM wrote a dense matrix
        if (gu.part.part) return cudaErrorInvalidValue;
        return launch(geglu_wide_kernel, dim3(M), dim3(1024), 0, st, pdl, gu, F, bfrag, M);
    }
    const int ng = (F + 127) / 128 * 2;
    return launch(geglu_kernel, dim3(grid_for_warps(M * ng)), dim3(256), 0, st, pdl, gu, F, bfrag, M);
}
