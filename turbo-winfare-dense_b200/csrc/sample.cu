// Device-side token sampling: the reference's sample_token (src/sampling.cpp:92-169) over a
// logits row in device memory, so the non-speculative sampled loop needs no logits readback.
//
// The reference's steps, and how each is done here:
//   * greedy (temperature <= 0): argmax, ties to the lowest index;
//   * max logit, then the full-distribution denominator  total = sum_v exp((double)l_v - max);
//   * a shortlist of the `want` largest logits (ties to the lower index), want = top_k, or 256
//     when top_k is 0, sorted descending;
//   * top-p over the shortlist with the true probabilities exp(l - max) / total, then top-k,
//     cut >= 1;
//   * q_i = exp((l_i - max) / T) over the survivors, r = uniform(xorshift64*) * sum q, and the
//     first survivor whose running sum reaches r.
//
// Kernel 1, one CTA per 4096-logit chunk: the chunk is bitonic-sorted in shared memory on a
// 64-bit key (order-preserving logit bits << 32 | ~index, so a larger key is a larger logit or,
// for equal logits, a lower index) and its 256 largest keys are kept, together with its maximum.
// Kernel 2, one CTA per chunk: every CTA forms the global maximum and its chunk's share of the
// denominator (fp64, fixed order); the last CTA to arrive adds the shares in chunk order, merges
// the sorted chunk lists into the global shortlist with one warp, and runs the short sequential
// tail (top-p scan, survivor weights, the draw) exactly as the reference orders it. The
// shortlist, the cut and the draw are therefore the reference's; only the denominator's
// summation order differs (chunked rather than one running sum), which can move a top-p cut or
// a draw only when it falls within a few units in the last place of a double of a boundary.
#include <cuda_runtime.h>

#include <cmath>
#include <algorithm>
#include <cstdint>

#include "kernels.h"

namespace g4b {

constexpr int kSampleChunk = 4096;   // logits per CTA in kernel 1
constexpr int kSampleKeep = 256;     // shortlist bound (the reference's kMaxTopK)
constexpr int kSampleMaxChunks = 64; // vocabularies up to 262144

struct SampleWork {
    unsigned long long cand[kSampleMaxChunks][kSampleKeep];
    float chunk_max[kSampleMaxChunks];
    double share[kSampleMaxChunks];
    unsigned arrived;
    unsigned token;
};

__device__ __forceinline__ unsigned long long sample_key(float l, unsigned i) {
    uint32_t u = __float_as_uint(l == 0.0f ? 0.0f : l);  // -0 and +0 compare equal in the reference
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (0xFFFFFFFFu - i);
}
__device__ __forceinline__ float key_logit(unsigned long long k) {
    const uint32_t o = (uint32_t)(k >> 32);
    return __uint_as_float((o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o);
}
__device__ __forceinline__ unsigned key_index(unsigned long long k) { return 0xFFFFFFFFu - (uint32_t)k; }

// xorshift64* and its 24-bit uniform (src/sampling.cpp:16-28).
__device__ __forceinline__ float next_uniform(unsigned long long& s) {
    s ^= s >> 12;
    s ^= s << 25;
    s ^= s >> 27;
    const unsigned long long r = s * 0x2545F4914F6CDD1DULL;
    return (float)((r >> 40) & 0xFFFFFF) / 16777216.0f;
}

__global__ void __launch_bounds__(1024) sample_select_kernel(const float* __restrict__ logits, int V,
                                                             SampleWork* w) {
    __shared__ unsigned long long key[kSampleChunk];
    const int c = blockIdx.x, base = c * kSampleChunk;
    const int n = min(kSampleChunk, V - base);
    for (int i = threadIdx.x; i < kSampleChunk; i += blockDim.x)
        key[i] = i < n ? sample_key(logits[base + i], (unsigned)(base + i)) : 0ull;
    if (c == 0 && threadIdx.x == 0) w->arrived = 0;
    __syncthreads();
    // Bitonic sort, descending.
    for (int k = 2; k <= kSampleChunk; k <<= 1)
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < kSampleChunk; i += blockDim.x) {
                const int p = i ^ j;
                if (p > i) {
                    const unsigned long long a = key[i], b = key[p];
                    const bool desc = (i & k) == 0;
                    if (desc ? a < b : a > b) {
                        key[i] = b;
                        key[p] = a;
                    }
                }
            }
            __syncthreads();
        }
    for (int i = threadIdx.x; i < kSampleKeep; i += blockDim.x) w->cand[c][i] = key[i];
    if (threadIdx.x == 0) w->chunk_max[c] = n > 0 ? key_logit(key[0]) : -INFINITY;
}

__global__ void __launch_bounds__(256) sample_finish_kernel(const float* __restrict__ logits, int V, int nchunks,
                                                            SampleWork* w, float temperature, float top_p,
                                                            int top_k, unsigned long long seed, unsigned* out) {
    __shared__ unsigned long long merged[kSampleKeep];
    __shared__ double red[256];
    __shared__ double ew[kSampleKeep];
    __shared__ float s_max;
    __shared__ bool s_last;
    __shared__ int s_cut;
    const int c = blockIdx.x, tid = threadIdx.x, lane = tid & 31;

    if (temperature <= 0.0f) {  // greedy: the largest key overall
        if (c != 0) return;
        if (tid < 32) {
            unsigned long long best = 0;
            for (int b = lane; b < nchunks; b += 32) best = max(best, w->cand[b][0]);
            for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xFFFFFFFFu, best, o));
            if (lane == 0) {
                w->token = key_index(best);
                if (out) *out = key_index(best);
            }
        }
        return;
    }

    if (tid == 0) {
        float m = w->chunk_max[0];
        for (int b = 1; b < nchunks; ++b) m = fmaxf(m, w->chunk_max[b]);
        s_max = m;
    }
    __syncthreads();
    const double mx = (double)s_max;
    // This chunk's share of the denominator: a fixed per-thread order, then a fixed tree.
    double s = 0.0;
    const int base = c * kSampleChunk, n = min(kSampleChunk, V - base);
    for (int i = tid; i < n; i += blockDim.x) s += exp((double)logits[base + i] - mx);
    red[tid] = s;
    __syncthreads();
    for (int h = blockDim.x >> 1; h > 0; h >>= 1) {
        if (tid < h) red[tid] += red[tid + h];
        __syncthreads();
    }
    if (tid == 0) {
        w->share[c] = red[0];
        __threadfence();
        s_last = atomicAdd(&w->arrived, 1u) == (unsigned)nchunks - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();

    // Shortlist: the chunks' sorted lists come into shared memory, then warp 0 merges them
    // (each lane owns chunks lane and lane + 32).
    extern __shared__ unsigned long long cand_s[];  // [nchunks][kSampleKeep]
    for (int i = tid; i < nchunks * kSampleKeep; i += blockDim.x) cand_s[i] = __ldcg(&w->cand[0][0] + i);
    __syncthreads();
    const int want = top_k > 0 ? min(top_k, V) : min(kSampleKeep, V);
    if (tid < 32) {
        int hp[2] = {0, 0};
        unsigned long long hk[2];
        for (int r = 0; r < 2; ++r) {
            const int b = lane + 32 * r;
            hk[r] = b < nchunks ? cand_s[b * kSampleKeep] : 0ull;
        }
        for (int i = 0; i < want; ++i) {
            const int rb = hk[1] > hk[0] ? 1 : 0;
            unsigned long long best = hk[rb];
            for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xFFFFFFFFu, best, o));
            if (lane == 0) merged[i] = best;
            if (best != 0ull && hk[rb] == best) {  // keys are unique: exactly one lane advances
                const int b = lane + 32 * rb;
                ++hp[rb];
                hk[rb] = hp[rb] < kSampleKeep ? cand_s[b * kSampleKeep + hp[rb]] : 0ull;
            }
        }
    }
    __syncthreads();
    double total = 0.0;
    if (tid == 0)
        for (int b = 0; b < nchunks; ++b) total += __ldcg(&w->share[b]);
    // Top-p with the true probabilities, in shortlist order (src/sampling.cpp:132-140).
    if (tid < want) ew[tid] = exp((double)key_logit(merged[tid]) - mx);
    __syncthreads();
    if (tid == 0) {
        int cut = want;
        if (top_p < 1.0f) {
            double run = 0.0;
            for (int i = 0; i < want; ++i) {
                run += ew[i] / total;
                if (run >= (double)top_p) {
                    cut = i + 1;
                    break;
                }
            }
        }
        if (top_k > 0) cut = min(cut, top_k);
        s_cut = max(1, cut);
    }
    __syncthreads();
    const int cut = s_cut;
    // Survivor weights with the temperature, then the draw (src/sampling.cpp:146-168).
    if (tid < cut) ew[tid] = exp(((double)key_logit(merged[tid]) - mx) / (double)temperature);
    __syncthreads();
    if (tid == 0) {
        double denom = 0.0;
        for (int i = 0; i < cut; ++i) denom += ew[i];
        unsigned long long st = seed;
        const double r = (double)next_uniform(st) * denom;
        double acc = 0.0;
        unsigned tok = key_index(merged[cut - 1]);
        for (int i = 0; i < cut; ++i) {
            acc += ew[i];
            if (acc >= r) {
                tok = key_index(merged[i]);
                break;
            }
        }
        w->token = tok;
        if (out) *out = tok;
    }
}

// Repetition penalty (apply_repetition_penalty, src/sampling.cpp:74-90) on the device. The
// reference walks the history in order and, for every occurrence of an id, divides a positive
// logit by the penalty (or multiplies a negative one), clamping to +-0.9999 * softcap. Each id's
// value depends only on its own occurrences, so applying the step count[id] times to every
// distinct id gives the same floats in any id order.
__global__ void rep_penalty_kernel(float* __restrict__ logits, const uint32_t* __restrict__ count,
                                   const uint32_t* __restrict__ ids, const int* __restrict__ n, float penalty,
                                   float limit) {
    const int nd = *n;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < nd; i += gridDim.x * blockDim.x) {
        const uint32_t id = ids[i];
        float v = logits[id];
        for (uint32_t k = count[id]; k > 0; --k) {
            v = (v > 0.0f) ? (v / penalty) : (v * penalty);
            if (limit > 0.0f) v = fminf(fmaxf(v, -limit), limit);
        }
        logits[id] = v;
    }
}

// Adds tokens to the history counts; an id seen for the first time joins the distinct list.
__global__ void rep_append_kernel(uint32_t* __restrict__ count, uint32_t* __restrict__ ids, int* __restrict__ n,
                                  const uint32_t* __restrict__ toks, int ntok, int V) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < ntok; i += gridDim.x * blockDim.x) {
        const uint32_t id = toks[i];
        if (id >= (uint32_t)V) continue;  // out-of-range ids are ignored, as in the reference
        if (atomicAdd(&count[id], 1u) == 0u) ids[atomicAdd(n, 1)] = id;
    }
}

}  // namespace g4b

using namespace g4b;

cudaError_t g4b_rep_penalty(float* logits, const uint32_t* count, const uint32_t* ids, const int* n, float penalty,
                            float limit, cudaStream_t st) {
    rep_penalty_kernel<<<64, 256, 0, st>>>(logits, count, ids, n, penalty, limit);
    return cudaGetLastError();
}

cudaError_t g4b_rep_append(uint32_t* count, uint32_t* ids, int* n, const uint32_t* toks, int ntok, int V,
                           cudaStream_t st) {
    if (ntok <= 0) return cudaSuccess;
    rep_append_kernel<<<std::min(148, (ntok + 255) / 256), 256, 0, st>>>(count, ids, n, toks, ntok, V);
    return cudaGetLastError();
}

size_t g4b_sample_workspace_bytes() { return sizeof(SampleWork); }

cudaError_t g4b_sample_launch(const float* logits, int V, float temperature, float top_p, int top_k,
                              unsigned long long seed, void* work, unsigned* out, cudaStream_t st) {
    if (V < 1 || V > kSampleChunk * kSampleMaxChunks || top_k < 0 || top_k > kSampleKeep || !work)
        return cudaErrorInvalidValue;
    const int nchunks = (V + kSampleChunk - 1) / kSampleChunk;
    SampleWork* w = static_cast<SampleWork*>(work);
    sample_select_kernel<<<nchunks, 1024, 0, st>>>(logits, V, w);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const size_t smem = (size_t)nchunks * kSampleKeep * sizeof(unsigned long long);
    static bool attr_set = false;
    if (!attr_set) {
        e = cudaFuncSetAttribute(sample_finish_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 kSampleMaxChunks * kSampleKeep * (int)sizeof(unsigned long long));
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    sample_finish_kernel<<<nchunks, 256, smem, st>>>(logits, V, nchunks, w, temperature, top_p, top_k, seed, out);
    return cudaGetLastError();
}
