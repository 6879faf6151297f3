/* CPU restatement of the reference's speculative-decode path, in plain C.
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker for the B200 engine. Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg load it. Each function cites the
 * reference file:line it restates. Its forward pass is pinned bit-for-bit against the
 * reference's own src/cpu_reference.cpp (built into oracle/_ref) on the same containers.
 *
 * Differences from the reference's CPU oracle, all additive:
 *   - the KV cache can be truncated (the reference can only append, so callers replay);
 *   - KV rounding mode is selectable (FP16 = the reference; BF16 for the bf16-KV config);
 *   - the speculative loop of src/runner.cpp:2120-2347 is restated over this forward pass;
 *   - per-layer FFN widths, per-layer inputs and layers that read another layer's K/V (the
 *     E2B/E4B architecture) follow the reference's GPU runner (src/runner.cpp:271-370, 960-1085,
 *     1240-1336, 1745-1825), which is the only C++ code of the reference that runs them. That
 *     path is pinned against the reference's NumPy forward pass (tools/numpy_reference.py) on
 *     synthetic checkpoints; a container without these features takes the unchanged path above.
 *
 * The MTP drafter's restatement (g4o_mtp_*) is the exception to the pinning: parity unpinned.
 */
#ifndef G4D_ORACLE_H
#define G4D_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct g4o_model g4o_model;

typedef struct {
    float temperature;        /* 0 = greedy */
    float top_p;              /* 1 = off */
    int top_k;                /* 0 = off */
    float repetition_penalty; /* 1 = off */
    int has_seed;
    uint64_t seed;
} g4o_sampling;

enum { G4O_KV_FP16 = 0, G4O_KV_BF16 = 1, G4O_KV_FP32 = 2 };

const char* g4o_last_error(void);

/* Opens a .g4dense v3 container. max_ctx bounds the KV length. cache_dequant != 0 keeps
 * fp32 copies of every matrix (fast for small models; the reference re-dequantizes). */
g4o_model* g4o_open(const char* path, int kv_mode, uint32_t max_ctx, int cache_dequant);
void g4o_close(g4o_model* m);
/* out[0..11] = num_layers, d_model, d_ff, q_heads, kv_heads, head_dim, vocab, window,
 *              global_head_dim, global_kv_heads, low 32 bits of global mask, high 32 bits */
void g4o_info(const g4o_model* m, uint32_t* out);
uint32_t g4o_length(const g4o_model* m);
void g4o_truncate(g4o_model* m, uint32_t len);
/* Forward one token at position `pos` (== current length). Writes vocab logits (softcapped)
 * and, when hidden_out is non-null, the final normed hidden state [d_model]. */
int g4o_forward(g4o_model* m, uint32_t token, uint32_t pos, float* logits, float* hidden_out);

/* ---- kernel-level restatements ---- */
float g4o_bf16_to_f32(uint16_t v);
uint16_t g4o_f32_to_bf16_rne(float f);
float g4o_round_f16(float f);
float g4o_round_bf16(float f);
float g4o_gelu_tanh(float x);
/* out[m][r] = sum_c (q*s+b) * x[m][c]; sequential fp32 sum per row, as cpu_reference gemv. */
void g4o_int4_gemm(const uint32_t* W, const uint16_t* S, const uint16_t* B, uint32_t rows,
                   uint32_t cols, const float* x, uint32_t M, float* out);
void g4o_attn_gate(const float* ctx, const float* gate, float* out, uint32_t n);
void g4o_int8_gemv(const uint32_t* W, const uint16_t* S, const uint16_t* B, uint32_t rows,
                   uint32_t cols, const float* x, float* out);
void g4o_rmsnorm(const float* x, const uint16_t* w_bf16, uint32_t n, float eps, float* out);
/* Multi-row GQA attention over an absolute-position cache (no ring):
 * q [M][qh*hd], K/V [n_keys][kvh*hd]; row m sees keys [first_m, n_pos+m) where
 * first_m = (window && n_pos+m > window) ? n_pos+m-window : 0. out [M][qh*hd]. */
void g4o_attention(const float* q, const float* K, const float* V, uint32_t M, uint32_t qh,
                   uint32_t kvh, uint32_t hd, uint32_t n_pos, uint32_t window, float scale,
                   float* out);

/* ---- MTP "assistant" drafter (.g4mtp v1; src/mtp_runner.cpp) ----
 * PARITY UNPINNED: the reference runs its MTP drafter only as Vulkan compute and has no CPU
 * implementation, golden vectors or known answers for it, so this restatement of
 * src/mtp_runner.cpp:263-843 is checked against nothing of the reference's own. */
typedef struct g4o_mtp g4o_mtp;
g4o_mtp* g4o_mtp_open(const char* path);
void g4o_mtp_close(g4o_mtp* m);
/* out[0..11] = num_layers, backbone, hidden, intermediate, vocab, q_heads, kv_heads, head_dim,
 *              global_head_dim, global_kv_heads, sliding_window, global mask (low 32 bits) */
void g4o_mtp_info(const g4o_mtp* m, uint32_t* out);
/* k draft tokens (and, if out_logits is non-null, their [k][vocab] logits) from the target's
 * final normed hidden state, the token at position context_length - 1 and the target's KV of
 * positions below it. The target must hold at least context_length - 1 positions. */
int g4o_mtp_draft(const g4o_mtp* mtp, const g4o_model* target, const float* target_hidden, uint32_t seed_token,
                  uint32_t context_length, uint32_t k, const g4o_sampling* sp, uint32_t* out_tokens,
                  float* out_logits);

/* ---- sampling / acceptance (src/sampling.cpp, src/speculator.cpp) ---- */
uint64_t g4o_splitmix64(uint64_t x);
uint64_t g4o_seed_for(const g4o_sampling* p, int position);
int g4o_validate_sampling(const g4o_sampling* p);
uint32_t g4o_sample_token(const float* logits, uint32_t vocab, const g4o_sampling* p, uint64_t seed);
uint32_t g4o_argmax(const float* logits, uint32_t vocab);
int g4o_evaluate_verification(const uint32_t* drafts, int k, const float* target_logits,
                              int n_target, uint32_t vocab, const g4o_sampling* p,
                              uint64_t base_seed, const float* draft_logits,
                              uint32_t* out_tokens, uint32_t* num_accepted);
/* std::mt19937_64 + uniform_real_distribution<float>(0,1) as libstdc++ draws them. */
void g4o_mt64_seed(uint64_t* state /*313 words*/, uint64_t seed);
float g4o_mt64_uniform_float(uint64_t* state);

/* ---- the decode loop (src/runner.cpp:2120-2347) ----
 * Same contract as oracle/ref_driver.cpp's ref_spec_generate. replay_stream (may be null)
 * switches the drafter to the config-3 "oracle drafter": at history length n it proposes
 * replay_stream[n - n_prompt] unless a seeded coin with probability mismatch_rate replaces
 * it by a different id. */
int g4o_spec_generate(g4o_model* target, g4o_model* draft, const uint32_t* prompt, int n_prompt,
                      int max_tokens, int verify_width, const g4o_sampling* p,
                      double gate_min_accept, int gate_window, int64_t stop_id,
                      const uint32_t* replay_stream, int replay_len, double mismatch_rate,
                      uint64_t mismatch_seed, uint32_t* out_tokens, int* round_info,
                      int max_rounds, int* n_rounds);

#ifdef __cplusplus
}
#endif
#endif
