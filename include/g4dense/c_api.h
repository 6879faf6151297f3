/* C ABI of the B200 speculative-decode engine (libg4dense_b200.so).
 *
 * The first block is the reference's C API, declaration for declaration
 * (include/g4dense/c_api.h:18-49 of the reference): same names, argument meanings, struct
 * layout, ownership and error behaviour (nullptr / -1 with g4dense_engine_last_error set;
 * returned strings stay valid until the next call on the same handle). A binding written
 * against the reference links against this library unchanged.
 *
 * The second block is additive: generation from token ids, speculation / tensor parallelism /
 * synthetic weights through g4dense_engine_create_ex, and the tokenizer on its own
 * (g4dense_tokenizer_*, the reference's Tokenizer / IncrementalDetokenizer /
 * StreamingStopMatcher), all without changing any existing signature.
 */
#ifndef G4DENSE_C_API_H
#define G4DENSE_C_API_H

#include <stddef.h>

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
/* Text generation (src/c_api.cpp:84-112): the prompt becomes one user turn of the chat
 * template, is encoded without a second <bos> and decoded with temperature 0.2, top_p 0.95,
 * top_k 64 and max_tokens (512 when <= 0), stopping after a tokenizer stop id
 * (src/runner.cpp:2060-2347). Returns the concatenated decode_single pieces of the emitted
 * tokens (the stop token's included; "" for special tokens). Needs the engine's tokenizer
 * (G4DenseEngineConfig.tokenizer_path, else $G4DENSE_TOKENIZER, else tokenizer.json beside the
 * container or in the working directory); without one, nullptr with last_error set. */
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

/* src/c_api.cpp:121-162. As the reference does, the messages_json text itself is the user
 * turn of the chat template (it is not parsed into messages); opts as given (NULL: the
 * runner's defaults). on_token receives each emitted token with its decode_single piece;
 * returning 0 stops generation. Returns the concatenated pieces, as g4dense_engine_generate. */
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
    const char* tokenizer_path;  /* tokenizer.json for the text entry points, or NULL to look for
                                    $G4DENSE_TOKENIZER, then tokenizer.json beside the container,
                                    then in the working directory (none found: text calls fail) */
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
/* ForwardRunner::generate(prompt, options) (src/runner.cpp:2060-2347) with the choice the
 * reference leaves to GenerationOptions::use_chat_template (include/g4dense/runner.hpp:50):
 * use_chat_template != 0 wraps `prompt` in one user turn and encodes it without <bos>;
 * 0 encodes it as given with <bos>. Otherwise as g4dense_engine_generate_ex. */
G4DENSE_API const char* g4dense_engine_generate_text(void* handle, const char* prompt, int use_chat_template,
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

/* ---- tokenizer (include/g4dense/tokenizer.hpp, include/g4dense/detokenizer.hpp) ----------
 * Strings returned by these calls stay valid until the next call on the same object; byte
 * lengths are written to *out_len (when non-NULL) because decoded text may hold NUL bytes. */

/* Tokenizer::load_vocabulary(path) then set_architecture(arch): arch 0 = Gemma-4,
 * 1 = Muse-Glimmer (ModelArch, include/g4dense/format.hpp:114-117). nullptr on error. */
G4DENSE_API void* g4dense_tokenizer_open(const char* tokenizer_json_path, int arch);
/* The tokenizer an engine loaded (owned by the engine), or nullptr when it has none. */
G4DENSE_API void* g4dense_engine_tokenizer(void* handle);
G4DENSE_API void g4dense_tokenizer_destroy(void* tok);
/* Tokenizer::encode (src/tokenizer.cpp:472-520) of text[0..len). Writes up to `cap` ids and
 * returns the full count (call again with a larger buffer when it exceeds cap), -1 on error. */
G4DENSE_API int g4dense_tokenizer_encode(void* tok, const char* text, size_t len, int add_bos, unsigned int* out,
                                         int cap);
/* Tokenizer::decode / decode_single (src/tokenizer.cpp:526-632). */
G4DENSE_API const char* g4dense_tokenizer_decode(void* tok, const unsigned int* ids, int n, int skip_special,
                                                 size_t* out_len);
G4DENSE_API const char* g4dense_tokenizer_decode_single(void* tok, unsigned int id, int skip_special,
                                                        size_t* out_len);
/* Tokenizer::apply_chat_template (src/tokenizer.cpp:638-672) of a JSON array of
 * {"role": ..., "content": ...} objects. nullptr on error (malformed JSON, a Gemma-4 system
 * message that is not first). */
G4DENSE_API const char* g4dense_tokenizer_chat_template(void* tok, const char* messages_json);
/* out[0..6) = bos, eos, pad, unk, end_of_turn, vocab_size; returns 0 or -1. */
G4DENSE_API int g4dense_tokenizer_special_ids(void* tok, unsigned int* out6);
/* Writes up to cap stop ids (Tokenizer::stop_token_ids); returns their count. */
G4DENSE_API int g4dense_tokenizer_stop_ids(void* tok, unsigned int* out, int cap);
/* 1 when `id` is a byte-fallback token (*value = its byte), else 0. */
G4DENSE_API int g4dense_tokenizer_byte_value(void* tok, unsigned int id, unsigned char* value);
/* 1 when `id` is marked special in added_tokens, else 0. */
G4DENSE_API int g4dense_tokenizer_is_special(void* tok, unsigned int id);

/* IncrementalDetokenizer (src/detokenizer.cpp:7-40) over a tokenizer that must outlive it. */
G4DENSE_API void* g4dense_detokenizer_create(void* tok, int skip_special);
G4DENSE_API const char* g4dense_detokenizer_push(void* detok, unsigned int id, size_t* out_len);
G4DENSE_API const char* g4dense_detokenizer_finish(void* detok, size_t* out_len);
G4DENSE_API void g4dense_detokenizer_destroy(void* detok);

/* StreamingStopMatcher (src/detokenizer.cpp:44-101). */
G4DENSE_API void* g4dense_stop_matcher_create(const char* const* stops, int n);
G4DENSE_API const char* g4dense_stop_matcher_push(void* m, const char* text, size_t len, size_t* out_len);
G4DENSE_API const char* g4dense_stop_matcher_finish(void* m, size_t* out_len);
/* 1 once a stop string matched (*matched, when non-NULL, points at it), else 0. */
G4DENSE_API int g4dense_stop_matcher_stopped(void* m, const char** matched);
G4DENSE_API void g4dense_stop_matcher_destroy(void* m);

/* utf8_repair (src/tokenizer.cpp:563-598): appends the repaired prefix of in[0..len) and
 * returns it; *consumed = bytes of `in` used. The string stays valid until the next call on
 * this thread. */
G4DENSE_API const char* g4dense_utf8_repair(const char* in, size_t len, int flush_all, size_t* consumed,
                                            size_t* out_len);

/* Checks the header of the container at `path` against the file's size with the rules the
 * engine's loader applies (the reference's validate_header / validate_mtp_header,
 * src/format.cpp:6-130, plus what this engine needs to run the model). Needs no GPU and does not
 * read the payload. Returns 1 for a valid .g4dense, 2 for a valid .g4mtp, or -1 with every broken
 * rule in g4dense_engine_last_error(). */
G4DENSE_API int g4dense_container_validate(const char* path);

#ifdef __cplusplus
}
#endif

#endif /* G4DENSE_C_API_H */
