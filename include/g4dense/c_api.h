/* C ABI of the B200 speculative-decode engine (libg4dense_b200.so).
 *
 * The first block is the reference's C API, declaration for declaration
 * (include/g4dense/c_api.h:18-49 of the reference): same names, argument meanings, struct
 * layout, ownership and error behaviour (nullptr / -1 with g4dense_engine_last_error set;
 * returned strings stay valid until the next call on the same handle). A binding written
 * against the reference links against this library unchanged.
 *
 * The second block is additive. The reference drives its engine with text through a
 * tokenizer; this path is driven by token ids, and speculation / tensor parallelism /
 * synthetic weights are enabled through g4dense_engine_create_ex without changing any
 * existing signature.
 */
#ifndef G4DENSE_C_API_H
#define G4DENSE_C_API_H

#ifdef __cplusplus
extern "C" {
#endif

#define G4DENSE_API __attribute__((visibility("default")))

/* ---- reference API (include/g4dense/c_api.h:18-49) ---------------------------------- */

/* Loads a .g4dense v3 container fully resident on the current CUDA device. Replaces
 * g4dense_engine_create (src/c_api.cpp:55-77). Returns nullptr on failure. */
G4DENSE_API void* g4dense_engine_create(const char* container_path);
/* src/c_api.cpp:79-82 */
G4DENSE_API void g4dense_engine_destroy(void* handle);
/* Text generation (src/c_api.cpp:84-112). This path has no tokenizer (the reference's
 * tokenizer.json is not part of it), so this returns nullptr with last_error set; use
 * g4dense_engine_generate_tokens. */
G4DENSE_API const char* g4dense_engine_generate(void* handle, const char* prompt, int max_tokens);
/* JSON telemetry with the reference's keys for the fields this engine measures
 * (src/c_api.cpp:114-119, src/telemetry.cpp:11-48). "{}" for a null handle. */
G4DENSE_API const char* g4dense_engine_get_telemetry(void* handle);

typedef struct {
    int max_tokens;
    float temperature;
    float top_p;
    int top_k;
    float repetition_penalty;
    int has_seed;
    unsigned long long seed;
    const char* system_prompt;
    const char* const* stop_strings;
    int stop_count;
    int tier_id;
} G4DenseGenerationOptions;

/* Defaults of src/c_api.cpp:40-53: 512 tokens, temperature 0.2, top_p 0.95, top_k 64. */
G4DENSE_API void g4dense_options_default(G4DenseGenerationOptions* out);

typedef int (*G4DenseTokenCallback)(void* user, int index, unsigned int token_id, const char* delta);

/* Chat-message generation (src/c_api.cpp:121-162). Text needs a tokenizer: returns nullptr
 * with last_error set, as g4dense_engine_generate does. */
G4DENSE_API const char* g4dense_engine_generate_ex(void* handle, const char* messages_json,
                                                   const G4DenseGenerationOptions* opts,
                                                   G4DenseTokenCallback on_token, void* user);

/* 0 = max tokens, 1 = stop token, 2 = callback stop, 3 = cancelled (g4dense_engine_stop). */
G4DENSE_API int g4dense_engine_last_stop_reason(void* handle);
/* Thread-local message of the last failing call (src/c_api.cpp:28-31). */
G4DENSE_API const char* g4dense_engine_last_error(void);
/* Memory tiers are an APU residency concept (src/c_api.cpp:164-184); everything is resident
 * here, so any tier id >= 0 succeeds (0) and negative ids fail (-1). */
G4DENSE_API int g4dense_engine_switch_tier(void* handle, int tier_id);
/* Requests cancellation of the generation running on `handle` (the reference's is a no-op,
 * src/c_api.cpp:186-188); takes effect before the next verify round. */
G4DENSE_API void g4dense_engine_stop(void* handle);

/* ---- additive API --------------------------------------------------------------------- */

typedef struct {
    const char* container_path;  /* target .g4dense, or NULL with synthetic_preset */
    const char* synthetic_preset;/* "gemma4-31b", "config0-target", ... (device-generated
                                    weights with the container's value distributions) */
    unsigned long long synthetic_seed;
    int synthetic_centered;      /* zero-mean groups (test aid; see container writer) */
    const char* draft_path;      /* drafter .g4dense, or NULL */
    const char* draft_preset;    /* "gemma4-e2b", "config0-draft", or NULL */
    unsigned long long draft_seed;
    int draft_k;                 /* verify width K (K-1 drafts); 0 disables speculation */
    int max_context;             /* KV capacity of full-attention layers (default 4096) */
    int kv_bf16;                 /* 1: bf16 KV instead of the reference's FP16 */
    int tp_rank, tp_size;        /* tensor parallelism (1 = off) */
    const void* nccl_unique_id;  /* 128-byte ncclUniqueId shared by all ranks when tp_size > 1 */
    int device;                  /* CUDA device ordinal (-1 = current) */
    double gate_min_accept;      /* adaptive gate (default 0.45 over 24 drafts) */
    int gate_window;
} G4DenseEngineConfig;

G4DENSE_API void g4dense_config_default(G4DenseEngineConfig* out);
G4DENSE_API void* g4dense_engine_create_ex(const G4DenseEngineConfig* cfg);

/* Generation from token ids (the reference's generate() with use_chat_template = false,
 * include/g4dense/runner.hpp:50). Tokens are delivered through on_token (delta = "") and
 * the emitted ids can be read back with g4dense_engine_last_tokens. Returns a short JSON
 * summary string (valid until the next call on the handle) or nullptr on error. */
G4DENSE_API const char* g4dense_engine_generate_tokens(void* handle, const unsigned int* prompt_ids, int n_prompt,
                                                       const G4DenseGenerationOptions* opts,
                                                       G4DenseTokenCallback on_token, void* user);
/* Copies up to `cap` ids of the last generation into out; returns the count. */
G4DENSE_API int g4dense_engine_last_tokens(void* handle, unsigned int* out, int cap);
/* ForwardRunner::forward_batch (include/g4dense/runner.hpp:110-111): one pass over `batch`
 * positions from base_position; out_logits (host, may be NULL) receives the last row's
 * softcapped logits, or all rows' when all_positions != 0. 1..16 rows run the verify pass;
 * 17..128 rows a tensor-core prefill chunk, which returns the last row only (all_positions
 * with more than 16 rows is an error). Returns 0 or -1. */
G4DENSE_API int g4dense_engine_forward_batch(void* handle, const unsigned int* token_ids, int batch,
                                             int base_position, float* out_logits, int all_positions);
/* Greedy decoding knobs beyond G4DenseGenerationOptions (additive): stop token id, and the
 * config-3 replay drafter (target stream + injected mismatch rate). */
G4DENSE_API int g4dense_engine_set_decode_options(void* handle, long long stop_token, int draft_k,
                                                  const unsigned int* replay, int replay_len, double mismatch_rate,
                                                  unsigned long long mismatch_seed);
/* Non-speculative sampled decoding (temperature > 0, no repetition penalty) draws each token on
 * the device by default, as sample_token does on the host (src/sampling.cpp:92-169); on = 0
 * selects the host draw over a copied logits row. Additive; returns 0 or -1. */
G4DENSE_API int g4dense_engine_set_device_sampling(void* handle, int on);
/* MtpRunner::generate_draft_tokens (src/mtp_runner.cpp:263-843) with greedy drafting, for an
 * engine whose drafter is an MTP assistant (.g4mtp): k draft tokens from seed_token at position
 * context_length - 1, starting from row hidden_row of the target's final normed hidden states of
 * its last pass (the last prompt position after a prefill chunk of more than 16 rows is row 0;
 * after a pass of M <= 16 rows, row M - 1). out_logits (host, may be NULL) receives [k][vocab].
 * Additive; returns 0 or -1. */
G4DENSE_API int g4dense_engine_mtp_draft(void* handle, unsigned int seed_token, int context_length, int hidden_row,
                                         int k, unsigned int* out_tokens, float* out_logits);
/* DraftRuntime::generate_draft_tokens (src/draft_runtime.cpp:46-95) with greedy drafting, for an
 * engine with a separate drafter model: k chained one-row drafter steps (k <= 64) from `token` at
 * position `pos` over the drafter's current KV cache (each step writes its own position's K/V),
 * each step's argmax feeding the next. out_tokens receives the k drafts; out_logits (host, may be
 * NULL) each step's softcapped logits [k][vocab]. Additive; returns 0 or -1. */
G4DENSE_API int g4dense_engine_draft_steps(void* handle, unsigned int token, int pos, int k, unsigned int* out_tokens,
                                           float* out_logits);
/* Per-round (drafted, accepted, emitted) triples of the last speculative generation. */
G4DENSE_API int g4dense_engine_last_rounds(void* handle, int* out, int cap_triples);
G4DENSE_API int g4dense_nccl_unique_id(void* out128);
/* Statistics of the last generation: {emitted, decode device ms (CUDA events from the end of
 * prefill), ttft ms, total ms, drafted, accepted, rounds, gated steps, kernel launches,
 * host->device bytes, device->host bytes, decode wall ms}. Returns how many were written. */
G4DENSE_API int g4dense_engine_last_stats(void* handle, double* out, int n);
/* The adaptive drafting gate (src/runner.cpp:2188-2195): stop drafting once at least `window`
 * drafts have been made and fewer than min_accept of them were accepted; window < 0 disables
 * it. Defaults 0.45 / 24. */
G4DENSE_API int g4dense_engine_set_gate(void* handle, double min_accept, int window);
/* Device time (CUDA events) of one forward pass of `batch` rows at positions pos..pos+batch-1
 * on the target (which = 0) or the drafter (which = 1), averaged over `reps` back-to-back graph
 * replays; attention spans the pos earlier cache entries. batch 1..16 times a verify pass,
 * 17..128 a tensor-core prefill chunk. Overwrites those rows of the KV cache. which = 2 times one
 * step of an MTP drafter (batch 1) whose query attends the target's pos cached positions. -1 on
 * error. */
G4DENSE_API double g4dense_engine_time_pass(void* handle, int which, int batch, int pos, int reps);
/* Times every verify GEMM of one `batch`-row target pass, `reps` passes back to back, with
 * CUDA events; returns ms per pass (-1 on error), the pass's algorithmic GEMM bytes and the
 * GEMM launches per pass. A measurement hook for the verify-GEMM bandwidth metric. */
G4DENSE_API double g4dense_engine_profile_gemms(void* handle, int batch, int reps, unsigned long long* bytes,
                                                int* launches);

#ifdef __cplusplus
}
#endif

#endif /* G4DENSE_C_API_H */
