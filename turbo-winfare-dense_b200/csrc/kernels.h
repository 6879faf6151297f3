// Host-side launchers of the device kernels (internal to the library).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

#include "model_dev.h"

// ---- repack.cu
size_t g4b_qmat_bytes(int N, int K);
cudaError_t g4b_repack(const uint32_t* W, const uint16_t* S, const uint16_t* B, int N, int K, void* out,
                       cudaStream_t st);

// ---- rowops.cu
// x fp32 [M][ldx] (K used columns) -> B fragments for a K-column GEMM input (K padded to 128).
cudaError_t g4b_bfrag_from_f32(const float* x, int ldx, int M, int K, void* bfrag, cudaStream_t st, bool pdl);
cudaError_t g4b_embed_norm(const g4b::StepParams* sp, const uint32_t* ew, const uint16_t* es, const uint16_t* eb,
                           int V, int d, const uint16_t* w_in, float* h_out, void* bfrag, int M, cudaStream_t st,
                           bool pdl);
cudaError_t g4b_qkv_epi(const g4b::QkvEpiArgs& a, cudaStream_t st, bool pdl);
// MTP drafter step input [e(t) * sqrt(bb); h] -> B fragments (one row, K = 2 * bb); h from
// hidden[sp->aux] when hidden is set, else from the previous post-projection's output `post`.
cudaError_t g4b_mtp_input(const g4b::StepParams* sp, const uint32_t* ew, const uint16_t* es, const uint16_t* eb,
                          int V, int bb, const float* hidden, const g4b::GemmOut& post, void* bfrag, cudaStream_t st,
                          bool pdl);
cudaError_t g4b_geglu(const g4b::GemmOut& gu, int F, void* bfrag, int M, cudaStream_t st, bool pdl);
// Norm/residual epilogue (post-attention with out_scale = 1, post-FFN with the layer scalar):
// h_out = (h_in + rmsnorm(o)*w1) * out_scale; x = rmsnorm(h_out)*w2 -> B fragments.
// Under tensor parallelism (tg.n > 1) y is the rank-ordered sum of every rank's dense partial
// (TpGather); otherwise o's slots or dense matrix. w1 == nullptr adds o unnormalised and h_in ==
// nullptr starts from zero (h_out = o: a projection's output becoming the residual stream).
// x_out (optional) also receives x in fp32, [M - frag_row0][d].
cudaError_t g4b_rowepi(const g4b::GemmOut& o, const g4b::TpGather& tg, const float* h_in, float* h_out,
                       const uint16_t* w1, float out_scale, const uint16_t* w2, int d, void* bfrag, int M,
                       cudaStream_t st, bool pdl,
                       int frag_row0 = 0, float* x_out = nullptr);

// ---- attention.cu
// Attention of M rows over the KV ring; writes the output [M][qh*hd] as the o-projection's
// B fragments. One 8-CTA cluster per (KV head, 16 query rows), key splits combined in DSMEM.
cudaError_t g4b_attention(const g4b::AttnArgs& a, void* bfrag, cudaStream_t st, bool pdl);

namespace g4b {
// Long-context attention for full-attention layers with head_dim 512 and a bf16 KV cache
// (attn_lc.cu). attn_lc_groups is 0 where a batch of M rows cannot use it.
int attn_lc_groups(int M, int gqa);
void attn_lc_scratch(int qh, int kvh, size_t* part_bytes, size_t* ml_bytes);
cudaError_t make_kv_tmap(KvTmap* out, const uint16_t* ring, int hd, int kvh, int cap);
cudaError_t attention_lc(const AttnArgs& a, const KvTmap& k, const KvTmap& v, float* part, float2* ml, int* err,
                         void* bfrag, cudaStream_t st, bool pdl);
}  // namespace g4b

// ---- head.cu
struct HeadResult {
    int n_emit;          // tokens emitted by greedy acceptance (accepted drafts + 1)
    int n_accepted;      // drafts accepted
    uint32_t tokens[17]; // emitted ids
    uint32_t argmax[16]; // per-row greedy target token
};
int g4b_head_chunks(int V);
// Softcapped logits (written when `logits` is non-null) and per-chunk (max, global index =
// local index + v_off) into chunk_best [M][chunks].
cudaError_t g4b_head_chunks_launch(const g4b::GemmOut& lm, int V, int M, float softcap, float* logits, int ldl,
                                   float2* chunk_best, int v_off, cudaStream_t st, bool pdl);
// Per-row argmax (ties to the lowest index) and greedy acceptance of sp->tokens[1..M-1]
// against argmax[0..M-2]. With chain_out (drafter steps) the last row's argmax also becomes
// the next pass's input: sp->tokens[0] = t, sp->base_pos += M, chain_out[sp->draft_step++] = t.
// chunk_best holds nranks slices [M][nchunks] (tensor-parallel vocabulary ranges).
// tp_seq (tensor parallelism, else nullptr) counts completed passes for the peer-memory sums.
cudaError_t g4b_head_finalize(const float2* chunk_best, int nchunks, int nranks, int M, g4b::StepParams* sp,
                              HeadResult* res, uint32_t* chain_out, unsigned* tp_seq, cudaStream_t st, bool pdl,
                              bool advance_pos = true);

// ---- sample.cu: sample_token (src/sampling.cpp:92-169) over a device logits row. `work` is
// g4b_sample_workspace_bytes() of device memory, private to one stream at a time; the token is
// written to *out (device memory, may be null) and to the workspace.
size_t g4b_sample_workspace_bytes();
cudaError_t g4b_sample_launch(const float* logits, int V, float temperature, float top_p, int top_k,
                              unsigned long long seed, void* work, unsigned* out, cudaStream_t st);

// Repetition penalty on a device logits row from history counts (count [V], the distinct ids
// ids[0..*n)), and appending tokens (device ids) to those counts.
cudaError_t g4b_rep_penalty(float* logits, const uint32_t* count, const uint32_t* ids, const int* n, float penalty,
                            float limit, cudaStream_t st);
cudaError_t g4b_rep_append(uint32_t* count, uint32_t* ids, int* n, const uint32_t* toks, int ntok, int V,
                           cudaStream_t st);

// ---- side.cu: INT8 G64 GEMV (one row per warp) and the attention output gate
namespace g4b {
cudaError_t gemv_int8_launch(const uint8_t* W, const uint16_t* S, const uint16_t* B, const float* x, float* out,
                             int rows, int K, cudaStream_t st);
cudaError_t attn_gate_launch(const float* ctx, const float* gate, float* out, int n, int batch, int ctx_stride,
                             int gate_stride, int out_stride, cudaStream_t st);
}  // namespace g4b
