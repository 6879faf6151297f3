// LM head epilogue and on-device greedy acceptance.
//
// Restates, for the tied INT4 head (src/cpu_reference.cpp:635-665): logits = softcap(z) with
// softcap(z) = 30*tanh(z/30), then the greedy target token per row = argmax with ties to
// the LOWEST index (src/sampling.cpp:297-304, shaders/ArgmaxReduce.hlsl:15-62). The argmax is
// taken over the softcapped values, as the reference's sample_token sees them, so saturated
// ties resolve exactly as on the CPU.
//
// Greedy acceptance (src/speculator.cpp:53-69, 138-146): with the verify batch
// [pending, d1 .. d_{M-1}], draft d_{i+1} is accepted while it equals argmax(row i); the
// emitted tokens are argmax(row 0 .. row n_acc), i.e. the accepted drafts followed by the
// correction or bonus token.
#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"
#include "model_dev.h"

#include <algorithm>

namespace g4b {

constexpr int kHeadChunk = 4096;

__device__ __forceinline__ bool better(float v, uint32_t i, float bv, uint32_t bi) {
    return v > bv || (v == bv && i < bi);
}

// chunk_best[m][chunk] = {best softcapped logit, its GLOBAL vocabulary index (v + v_off)}.
__global__ void head_chunks_kernel(GemmOut lm, int V, int M, float softcap, float* logits, int ldl,
                                   float2* chunk_best, int v_off) {
    __shared__ float sv[32];
    __shared__ uint32_t si[32];
    pdl_enter();
    const int chunk = blockIdx.x, m = blockIdx.y;
    const int v0 = chunk * kHeadChunk, v1 = min(V, v0 + kHeadChunk);
    float bv = -INFINITY;
    uint32_t bi = 0xFFFFFFFFu;
    // Four 256-wide column blocks per batch; with split-K partials each block is its own row
    // group, and all of a batch's slot loads are issued together.
    for (int b0 = v0; b0 < v1; b0 += 4 * 256) {
        float z[4];
        if (lm.part.part) {
            const float* pj[4];
            int nsj[4], nsmax = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int v = b0 + j * 256 + threadIdx.x;
                const int crg = (b0 >> 8) + j;
                pj[j] = slot_base(lm.part, m, crg) + threadIdx.x;
                nsj[j] = v < v1 ? slot_count(lm.part, crg) : 0;
                nsmax = max(nsmax, nsj[j]);
            }
            slot_sums_each<4, 4>(pj, nsj, nsmax, z);
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int v = b0 + j * 256 + threadIdx.x;
                z[j] = v < v1 ? lm.y[(size_t)m * lm.ld + v] : 0.f;
            }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int v = b0 + j * 256 + threadIdx.x;
            if (v >= v1) continue;
            float zz = z[j];
            if (softcap > 0.f) zz = softcap * tanhf(zz / softcap);
            if (logits) logits[(size_t)m * ldl + v] = zz;
            const uint32_t gv = (uint32_t)(v + v_off);
            if (better(zz, gv, bv, bi)) { bv = zz; bi = gv; }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    if (lane == 0) { sv[wid] = bv; si[wid] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
            if (better(sv[w], si[w], bv, bi)) { bv = sv[w]; bi = si[w]; }
        chunk_best[(size_t)m * gridDim.x + chunk] = make_float2(bv, __uint_as_float(bi));
    }
}

// chunk_best is [nranks][M][nchunks] (one slice per tensor-parallel rank's vocabulary range);
// the order is total (value, then lowest index), so the result does not depend on the split.
__global__ void head_finalize_kernel(const float2* chunk_best, int nchunks, int nranks, int M, StepParams* sp,
                                     HeadResult* res, uint32_t* chain_out, unsigned* tp_seq, int advance_pos) {
    __shared__ uint32_t am[16];
    pdl_enter();
    const int lane = threadIdx.x & 31, m = threadIdx.x >> 5;
    if (m < M) {
        float bv = -INFINITY;
        uint32_t bi = 0xFFFFFFFFu;
        for (int c = lane; c < nranks * nchunks; c += 32) {
            const int r = c / nchunks;
            const float2 e = chunk_best[((size_t)r * M + m) * nchunks + c % nchunks];
            const uint32_t i = __float_as_uint(e.y);
            if (better(e.x, i, bv, bi)) { bv = e.x; bi = i; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) am[m] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int n_acc = 0;
        while (n_acc < M - 1 && sp->tokens[n_acc + 1] == am[n_acc]) ++n_acc;
        res->n_accepted = n_acc;
        res->n_emit = n_acc + 1;
        for (int i = 0; i <= n_acc; ++i) res->tokens[i] = am[i];
        for (int i = 0; i < M; ++i) res->argmax[i] = am[i];
        if (chain_out) {
            const uint32_t t = am[M - 1];
            chain_out[sp->draft_step] = t;
            sp->draft_step += 1;
            sp->tokens[0] = t;
            if (advance_pos) sp->base_pos += M;  // the MTP drafter keeps its position
        }
        if (tp_seq) *tp_seq += 1;  // the pass is complete on this rank
    }
}

}  // namespace g4b

using namespace g4b;

int g4b_head_chunks(int V) { return (V + kHeadChunk - 1) / kHeadChunk; }

cudaError_t g4b_head_chunks_launch(const GemmOut& lm, int V, int M, float softcap, float* logits, int ldl,
                                   float2* chunk_best, int v_off, cudaStream_t st, bool pdl) {
    // 256 threads, one column per thread per 256-wide block: blocks must align to row groups.
    static_assert(kHeadChunk % 256 == 0, "head chunk");
    return launch(head_chunks_kernel, dim3(g4b_head_chunks(V), M), dim3(256), 0, st, pdl, lm, V, M, softcap, logits,
                  ldl, chunk_best, v_off);
}

cudaError_t g4b_head_finalize(const float2* chunk_best, int nchunks, int nranks, int M, StepParams* sp,
                              HeadResult* res, uint32_t* chain_out, unsigned* tp_seq, cudaStream_t st, bool pdl,
                              bool advance_pos) {
    return launch(head_finalize_kernel, dim3(1), dim3(32 * 16), 0, st, pdl, chunk_best, nchunks, nranks, M, sp, res,
                  chain_out, tp_seq, advance_pos ? 1 : 0);
}
