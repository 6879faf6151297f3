// Row-wise kernels around the verify GEMM. Each consumes a GEMM's split-K slots (or an
// all-reduced matrix), applies the layer's elementwise/normalisation step in fp32 exactly as
// src/cpu_reference.cpp orders it, and produces the next GEMM's B fragments, so no
// activation is ever converted twice:
//   embed_norm   token gather x sqrt(d) (src/cpu_reference.cpp:260-291) + input RMSNorm
//   qkv_epi      q/k RMSNorm*w + NeoX RoPE, v unweighted RMSNorm (raw k on layers without
//                v_proj), K/V rounded and written to the ring (:398-498, QKVEpilogue.hlsl,
//                KVWrite.hlsl)
//   post_attn    h += rmsnorm(o)*w_post_attn; x = rmsnorm(h)*w_pre_ffn (:560-567)
//   geglu        gelu_tanh(gate) * up (:568-581, GeGLU.hlsl)
//   post_ffn     h = (h + rmsnorm(down)*w_post_ffn) * layer_scalar (:583-593), then the next
//                layer's input norm, or the final norm before the LM head (:610-629)
#include "bfrag.cuh"
#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"
#include "model_dev.h"

namespace g4b {

// FP16 round trip of the reference oracle (src/cpu_reference.cpp:51-84): round to nearest
// even for normal halves, values below the smallest normal half become signed zero, values
// at or above 2^16 become infinity. Returns the half's bit pattern.
__device__ __forceinline__ uint16_t f16_bits_like_reference(float f) {
    const uint32_t x = __float_as_uint(f);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const int e = (int)((x >> 23) & 0xFFu) - 127 + 15;
    const uint32_t man = x & 0x7FFFFFu;
    if (e <= 0) return (uint16_t)sign;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    const uint32_t round_bit = (man >> 12) & 1u;
    const uint32_t sticky = (man & 0xFFFu) != 0u;
    uint32_t v = sign | ((uint32_t)e << 10) | (man >> 13);
    if (round_bit && (sticky || (v & 1u))) ++v;
    return (uint16_t)v;
}

__device__ __forceinline__ uint16_t bf16_bits_rne(float f) {
    uint32_t u = __float_as_uint(f);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

__device__ __forceinline__ float kv_decode(uint16_t b, int bf16) {
    return bf16 ? __uint_as_float((uint32_t)b << 16) : __half2float(__ushort_as_half(b));
}

// 1 / sqrt(mean + eps) with IEEE sqrt and division, as the reference computes it.
__device__ __forceinline__ float inv_rms(float sumsq, int n) {
    return 1.0f / sqrtf(sumsq / (float)n + 1e-6f);
}

// Writes a full row x[0..K) (K a multiple of 64, in shared memory) as B fragments, one warp
// per 64-group.
__device__ __forceinline__ void row_to_bfrags(const float* xs, int K, int M, int m, void* bfrag, __half* stage) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int Kp = (K + 127) / 128 * 128;
    const BFragView v = bfrag_view(bfrag, Kp, M);
    for (int gi = warp; gi < Kp / 64; gi += nw) {
        const int k = gi * 64 + 2 * lane;
        const float x0 = k < K ? xs[k] : 0.f, x1 = k + 1 < K ? xs[k + 1] : 0.f;
        bfrag_store_group(v, M, m, gi, x0, x1, stage + warp * 128);
    }
}

// ---------------------------------------------------------------- embedding + input norm

__global__ void embed_norm_kernel(const StepParams* __restrict__ sp, const uint32_t* __restrict__ ew,
                                  const uint16_t* __restrict__ es, const uint16_t* __restrict__ eb, int V, int d,
                                  const uint16_t* __restrict__ w_in, float* __restrict__ h_out, void* bfrag, int M) {
    extern __shared__ float smem[];
    float* xs = smem;                                       // [d]
    __half* stage = reinterpret_cast<__half*>(xs + d);      // [warps][128]
    __shared__ float red[32];
    pdl_wait();
    const int m = blockIdx.x;
    uint32_t tok = sp->tokens[m];
    tok %= (uint32_t)V;
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
    row_to_bfrags(xs, d, M, m, bfrag, stage);
}

// ---------------------------------------------------------------- Q/K/V epilogue

// One block per (row m, head): heads [0, qh) are query heads, [qh, qh + kvh) KV heads.
__global__ void qkv_epi_kernel(QkvEpiArgs a) {
    extern __shared__ float smem[];
    float* xs = smem;          // [hd]
    float* vs = smem + a.hd;   // [hd]
    __shared__ float red[32];
    pdl_wait();
    const int m = blockIdx.x, head = blockIdx.y;
    const int hd = a.hd;
    const int pos = a.sp->base_pos + m;
    const int nq = a.qh * hd, nk = a.kvh * hd;
    const bool is_q = head < a.qh;
    const int kvh = head - a.qh;
    const int row0 = is_q ? head * hd : nq + kvh * hd;
    float ss = 0.f;
    for (int i = threadIdx.x; i < hd; i += blockDim.x) {
        const float v = gemm_out_get(a.qkv, m, row0 + i);
        xs[i] = v;
        ss += v * v;
    }
    const float r = inv_rms(block_sum(ss, red), hd);
    if (!is_q) {
        // V: unweighted norm of v_proj, or of the RAW k on layers without v_proj.
        float vss = 0.f;
        for (int i = threadIdx.x; i < hd; i += blockDim.x) {
            const float v = a.has_v ? gemm_out_get(a.qkv, m, nq + nk + kvh * hd + i) : xs[i];
            vs[i] = v;
            vss += v * v;
        }
        const float rv = inv_rms(block_sum(vss, red), hd);
        uint16_t* vd = a.v_ring + ((size_t)(pos % a.cap) * a.kvh + kvh) * hd;
        for (int i = threadIdx.x; i < hd; i += blockDim.x) {
            const float v = vs[i] * rv;
            vd[i] = a.kv_bf16 ? bf16_bits_rne(v) : f16_bits_like_reference(v);
        }
    }
    const uint16_t* w = is_q ? a.q_norm : a.k_norm;
    __syncthreads();
    for (int i = threadIdx.x; i < hd; i += blockDim.x) xs[i] = xs[i] * r * bf16_to_f32(w[i]);
    __syncthreads();
    // NeoX rotary on `rotated` pairs (i, i + hd/2).
    const int half = hd / 2;
    for (int p = threadIdx.x; p < a.rotated; p += blockDim.x) {
        const float freq = 1.0f / powf(a.theta, (float)(2 * p) / (float)hd);
        const float ang = (float)pos * freq;
        const float c = cosf(ang), s = sinf(ang);
        const float x0 = xs[p], x1 = xs[p + half];
        xs[p] = x0 * c - x1 * s;
        xs[p + half] = x0 * s + x1 * c;
    }
    __syncthreads();
    if (is_q) {
        float* qd = a.q_out + ((size_t)m * a.qh + head) * hd;
        for (int i = threadIdx.x; i < hd; i += blockDim.x) qd[i] = xs[i];
    } else {
        uint16_t* kd = a.k_ring + ((size_t)(pos % a.cap) * a.kvh + kvh) * hd;
        for (int i = threadIdx.x; i < hd; i += blockDim.x)
            kd[i] = a.kv_bf16 ? bf16_bits_rne(xs[i]) : f16_bits_like_reference(xs[i]);
    }
}

// ---------------------------------------------------------------- post-attention

__global__ void post_attn_kernel(GemmOut o, const float* __restrict__ h_in, float* __restrict__ h_out,
                                 const uint16_t* __restrict__ w_pa, const uint16_t* __restrict__ w_pf, int d,
                                 void* bfrag, int M) {
    extern __shared__ float smem[];
    float* ys = smem;                                   // [d]
    __half* stage = reinterpret_cast<__half*>(ys + d);  // [warps][128]
    __shared__ float red[32];
    pdl_wait();
    const int m = blockIdx.x;
    float ss = 0.f;
    for (int c = threadIdx.x; c < d; c += blockDim.x) {
        const float v = gemm_out_get(o, m, c);
        ys[c] = v;
        ss += v * v;
    }
    const float r1 = inv_rms(block_sum(ss, red), d);
    float ss2 = 0.f;
    for (int c = threadIdx.x; c < d; c += blockDim.x) {
        const float hn = h_in[(size_t)m * d + c] + ys[c] * r1 * bf16_to_f32(w_pa[c]);
        h_out[(size_t)m * d + c] = hn;
        ys[c] = hn;
        ss2 += hn * hn;
    }
    const float r2 = inv_rms(block_sum(ss2, red), d);
    for (int c = threadIdx.x; c < d; c += blockDim.x) ys[c] = ys[c] * r2 * bf16_to_f32(w_pf[c]);
    __syncthreads();
    row_to_bfrags(ys, d, M, m, bfrag, stage);
}

// ---------------------------------------------------------------- GeGLU

__device__ __forceinline__ float gelu_tanh_dev(float x) {
    const float k = 0.7978845608028654f;
    const float inner = k * (x + 0.044715f * x * x * x);
    return 0.5f * x * (1.0f + tanhf(inner));
}

// One warp per (row, 64-group) of the F-wide activation; gate rows [0, F), up rows [F, 2F).
__global__ void geglu_kernel(GemmOut gu, int F, void* bfrag, int M) {
    __shared__ __half stage[8][128];
    pdl_wait();
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int Fp = (F + 127) / 128 * 128;
    const int ng = Fp / 64;
    const BFragView v = bfrag_view(bfrag, Fp, M);
    for (int w = blockIdx.x * 8 + wib; w < M * ng; w += gridDim.x * 8) {
        const int m = w / ng, gi = w % ng;
        const int k = gi * 64 + 2 * lane;
        float x0 = 0.f, x1 = 0.f;
        if (k < F) x0 = gelu_tanh_dev(gemm_out_get(gu, m, k)) * gemm_out_get(gu, m, F + k);
        if (k + 1 < F) x1 = gelu_tanh_dev(gemm_out_get(gu, m, k + 1)) * gemm_out_get(gu, m, F + k + 1);
        bfrag_store_group(v, M, m, gi, x0, x1, stage[wib]);
    }
}

// ---------------------------------------------------------------- post-FFN

__global__ void post_ffn_kernel(GemmOut dn, const float* __restrict__ h_in, float* __restrict__ h_out,
                                const uint16_t* __restrict__ w_pffn, float layer_scalar,
                                const uint16_t* __restrict__ w_next, int d, void* bfrag, int M) {
    extern __shared__ float smem[];
    float* ys = smem;
    __half* stage = reinterpret_cast<__half*>(ys + d);
    __shared__ float red[32];
    pdl_wait();
    const int m = blockIdx.x;
    float ss = 0.f;
    for (int c = threadIdx.x; c < d; c += blockDim.x) {
        const float v = gemm_out_get(dn, m, c);
        ys[c] = v;
        ss += v * v;
    }
    const float r1 = inv_rms(block_sum(ss, red), d);
    float ss2 = 0.f;
    for (int c = threadIdx.x; c < d; c += blockDim.x) {
        const float hn = (h_in[(size_t)m * d + c] + ys[c] * r1 * bf16_to_f32(w_pffn[c])) * layer_scalar;
        h_out[(size_t)m * d + c] = hn;
        ys[c] = hn;
        ss2 += hn * hn;
    }
    const float r2 = inv_rms(block_sum(ss2, red), d);
    for (int c = threadIdx.x; c < d; c += blockDim.x) ys[c] = ys[c] * r2 * bf16_to_f32(w_next[c]);
    __syncthreads();
    row_to_bfrags(ys, d, M, m, bfrag, stage);
}

// ---------------------------------------------------------------- plain conversion

// x [M][ldx] fp32 -> B fragments. One warp per (row, 64-group); groups past K are zeros.
__global__ void bfrag_from_f32_kernel(const float* __restrict__ x, int ldx, int M, int K, void* bfrag) {
    __shared__ __half stage[8][128];
    pdl_wait();
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

cudaError_t g4b_qkv_epi(const QkvEpiArgs& a, cudaStream_t st, bool pdl) {
    return launch(qkv_epi_kernel, dim3(a.M, a.qh + a.kvh), dim3(128), (size_t)2 * a.hd * sizeof(float), st, pdl, a);
}

cudaError_t g4b_post_attn(const GemmOut& o, const float* h_in, float* h_out, const uint16_t* w_pa,
                          const uint16_t* w_pf, int d, void* bfrag, int M, cudaStream_t st, bool pdl) {
    const int th = 512;
    return launch(post_attn_kernel, dim3(M), dim3(th), row_smem(d, th), st, pdl, o, h_in, h_out, w_pa, w_pf, d,
                  bfrag, M);
}

cudaError_t g4b_geglu(const GemmOut& gu, int F, void* bfrag, int M, cudaStream_t st, bool pdl) {
    const int ng = (F + 127) / 128 * 2;
    return launch(geglu_kernel, dim3(grid_for_warps(M * ng)), dim3(256), 0, st, pdl, gu, F, bfrag, M);
}

cudaError_t g4b_post_ffn(const GemmOut& dn, const float* h_in, float* h_out, const uint16_t* w_pffn,
                         float layer_scalar, const uint16_t* w_next, int d, void* bfrag, int M, cudaStream_t st,
                         bool pdl) {
    const int th = 512;
    return launch(post_ffn_kernel, dim3(M), dim3(th), row_smem(d, th), st, pdl, dn, h_in, h_out, w_pffn,
                  layer_scalar, w_next, d, bfrag, M);
}
