// C-ABI driver over the REFERENCE's own CPU code, built into oracle/_ref/libg4ref.so.
//
// TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and bench.py's CPU
// baseline load it, and only as the checker. It links the unmodified reference sources
// (src/cpu_reference.cpp, src/format.cpp, src/sampling.cpp, src/speculator.cpp,
// src/tokenizer.cpp, src/detokenizer.cpp) compiled with oracle/shim/.
//
// The ref_tok_* / ref_detok_* / ref_stop_* functions expose the reference's Tokenizer,
// IncrementalDetokenizer and StreamingStopMatcher with the shapes of the engine's
// g4dense_tokenizer_* calls, so a test can drive both with the same inputs.
//
// What it restates (the reference has these only on its Vulkan path):
//   * ref_spec_generate: the decode loop of ForwardRunner::generate
//     (src/runner.cpp:2120-2347) -- prefill, the speculative round loop with its adaptive
//     gate, and the non-speculative loop -- driven over CpuReferenceRunner for both the
//     target and the drafter, with the reference's own SpeculativeCoordinator and
//     sample_token deciding every token.
//   * The drafter's bookkeeping from DraftRuntime (src/draft_runtime.cpp:46-103).
//
// CpuReferenceRunner appends K/V and cannot roll back (src/cpu_reference.cpp:497-498), so
// whenever a model must forget positions (rejected drafts) this driver rebuilds the runner
// and replays the surviving tokens. That is exact: the runner is a pure function of the
// token/position sequence it has been fed.
//
// One deliberate difference from DraftRuntime::accept (src/draft_runtime.cpp:97-103): when
// every draft of a round is accepted the reference marks the last draft as consumed although
// the drafter never forwarded it, so that KV slot is never written. Here (and in the B200
// engine) the drafter's consumed count is capped at what it actually forwarded, so the
// missing token is fed on the next round and the drafter's cache always matches its context.
#include "g4dense/cpu_reference.hpp"
#include "g4dense/detokenizer.hpp"
#include "g4dense/tokenizer.hpp"
#include "g4dense/sampling.hpp"
#include "g4dense/speculator.hpp"

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

using namespace g4dense;

namespace {

thread_local std::string g_err;

struct RefModel {
    std::string path;
    std::unique_ptr<CpuReferenceRunner> runner;
    uint32_t vocab{0};
    uint32_t fed{0};  // positions forwarded so far (the runner's KV length)

    void open() {
        CpuReferenceConfig cfg;
        cfg.container_path = path;
        runner = std::make_unique<CpuReferenceRunner>(cfg, nullptr);
        runner->initialize();
        fed = 0;
    }
    std::vector<float> forward(uint32_t tok, uint32_t pos) {
        if (pos != fed) throw std::runtime_error("ref driver: non-sequential position");
        auto l = runner->forward_single_token(tok, pos);
        ++fed;
        return l;
    }
    // Forget everything past `keep` positions by rebuilding and replaying.
    void truncate(const std::vector<uint32_t>& tokens, uint32_t keep) {
        if (keep == fed) return;
        open();
        for (uint32_t p = 0; p < keep; ++p) forward(tokens[p], p);
    }
};

SamplingParams make_params(float temperature, float top_p, int top_k, float rep, int has_seed,
                           uint64_t seed) {
    SamplingParams p;
    p.temperature = temperature;
    p.top_p = top_p;
    p.top_k = top_k;
    p.repetition_penalty = rep;
    p.has_seed = has_seed != 0;
    p.seed = seed;
    return p;
}

uint32_t header_vocab(const std::string& path) {
    FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) throw std::runtime_error("ref driver: cannot open " + path);
    G4DenseHeader h{};
    const size_t n = std::fread(&h, 1, sizeof(h), f);
    std::fclose(f);
    if (n != sizeof(h)) throw std::runtime_error("ref driver: short header");
    return h.vocab_size;
}

}  // namespace

extern "C" {

const char* ref_last_error(void) { return g_err.c_str(); }

void* ref_open(const char* path) {
    try {
        auto* m = new RefModel();
        m->path = path;
        m->vocab = header_vocab(m->path);
        m->open();
        return m;
    } catch (const std::exception& e) {
        g_err = e.what();
        return nullptr;
    }
}

void ref_close(void* h) { delete static_cast<RefModel*>(h); }

uint32_t ref_vocab(void* h) { return static_cast<RefModel*>(h)->vocab; }

// Forward one token at `pos` (must equal the number of positions already fed); writes
// vocab floats of softcapped logits. Returns 0, or -1 with ref_last_error set.
int ref_forward(void* h, uint32_t token, uint32_t pos, float* logits) {
    try {
        auto* m = static_cast<RefModel*>(h);
        auto l = m->forward(token, pos);
        std::memcpy(logits, l.data(), l.size() * sizeof(float));
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

int ref_reset(void* h) {
    try {
        static_cast<RefModel*>(h)->open();
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

uint64_t ref_splitmix64(uint64_t x) { return splitmix64(x); }

uint64_t ref_seed_for(float temperature, float top_p, int top_k, float rep, int has_seed,
                      uint64_t seed, int position) {
    return seed_for(make_params(temperature, top_p, top_k, rep, has_seed, seed), position);
}

// Returns the sampled id, or UINT32_MAX with ref_last_error set.
uint32_t ref_sample_token(const float* logits, uint32_t vocab, float temperature, float top_p,
                          int top_k, float rep, int has_seed, uint64_t seed, uint64_t rng_seed) {
    try {
        return sample_token(logits, vocab, make_params(temperature, top_p, top_k, rep, has_seed, seed),
                            rng_seed);
    } catch (const std::exception& e) {
        g_err = e.what();
        return UINT32_MAX;
    }
}

int ref_validate_sampling(float temperature, float top_p, int top_k, float rep) {
    try {
        validate_sampling(make_params(temperature, top_p, top_k, rep, 0, 0));
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

// SpeculativeCoordinator::evaluate_verification (src/speculator.cpp:34-153) over flat
// arrays: target_logits is [n_target][vocab], draft_logits is [k][vocab] or null.
// Writes the emitted tokens to out_tokens (capacity k+1) and returns their count; the
// number of accepted drafts goes to *num_accepted.
int ref_evaluate_verification(const uint32_t* drafts, int k, const float* target_logits,
                              int n_target, uint32_t vocab, float temperature, float top_p,
                              int top_k, float rep, int has_seed, uint64_t seed,
                              uint64_t base_seed, const float* draft_logits,
                              uint32_t* out_tokens, uint32_t* num_accepted) {
    try {
        SpeculativeCoordinator spec;
        std::vector<uint32_t> d(drafts, drafts + k);
        std::vector<const float*> per_pos;
        for (int i = 0; i < n_target; ++i) per_pos.push_back(target_logits + (size_t)i * vocab);
        std::vector<std::vector<float>> dl;
        if (draft_logits) {
            for (int i = 0; i < k; ++i)
                dl.emplace_back(draft_logits + (size_t)i * vocab, draft_logits + (size_t)(i + 1) * vocab);
        }
        auto ev = spec.evaluate_verification(
            d, per_pos, vocab, make_params(temperature, top_p, top_k, rep, has_seed, seed), base_seed, dl);
        for (size_t i = 0; i < ev.accepted_tokens.size(); ++i) out_tokens[i] = ev.accepted_tokens[i];
        *num_accepted = ev.num_accepted;
        return (int)ev.accepted_tokens.size();
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

// Restatement of ForwardRunner::generate (src/runner.cpp:2120-2347) over the reference's
// CPU oracle. `verify_width` is the reference's draft_k (K): K-1 drafts per round.
// draft_path may be null (no speculation). stop_id < 0 disables the stop-token check.
//
// Outputs: out_tokens[max_tokens] emitted ids; per verify round, round_info[3*r + {0,1,2}]
// = (drafted, accepted, emitted). Returns the number of emitted tokens and writes the
// number of speculative rounds to *n_rounds (gated single-token steps are not rounds).
int ref_spec_generate(const char* target_path, const char* draft_path, const uint32_t* prompt,
                      int n_prompt, int max_tokens, int verify_width, float temperature,
                      float top_p, int top_k, int has_seed, uint64_t seed, double gate_min_accept,
                      int gate_window, int64_t stop_id, uint32_t* out_tokens, int* round_info,
                      int max_rounds, int* n_rounds) {
    try {
        const SamplingParams sp = make_params(temperature, top_p, top_k, 1.0f, has_seed, seed);
        RefModel tgt;
        tgt.path = target_path;
        tgt.vocab = header_vocab(tgt.path);
        tgt.open();
        const uint32_t V = tgt.vocab;

        std::vector<uint32_t> history;
        for (int i = 0; i < n_prompt; ++i) {
            uint32_t t = prompt[i];
            if (t >= V) {
                // src/runner.cpp:2099-2109: small vocabularies wrap, large ones reject.
                if (V <= 4096) t %= V;
                else throw std::runtime_error("token id exceeds vocab");
            }
            history.push_back(t);
        }
        if (history.empty()) throw std::runtime_error("empty prompt");

        std::vector<float> logits;
        for (uint32_t p = 0; p < history.size(); ++p) logits = tgt.forward(history[p], p);

        int emitted = 0;
        int rounds = 0;
        auto is_stop = [&](uint32_t t) { return stop_id >= 0 && (int64_t)t == stop_id; };
        auto emit = [&](uint32_t t) { out_tokens[emitted++] = t; };

        if (draft_path && verify_width > 0) {
            RefModel drf;
            drf.path = draft_path;
            drf.vocab = header_vocab(drf.path);
            drf.open();
            size_t consumed = 0;  // DraftRuntime::consumed_

            const uint32_t K = std::min<uint32_t>((uint32_t)verify_width, 8u);
            SpeculativeCoordinator spec;
            uint32_t drafted_total = 0, accepted_total = 0;
            bool drafting = true;

            uint32_t pending =
                sample_token(logits.data(), V, sp, seed_for(sp, (int)(history.size() - 1)));
            history.push_back(pending);
            emit(pending);
            if (is_stop(pending)) return emitted;

            while (emitted < max_tokens) {
                if (!drafting) {
                    // Gated: one target pass per token (src/runner.cpp:2219-2237).
                    auto l = tgt.forward(pending, (uint32_t)(history.size() - 1));
                    const uint32_t next = sample_token(l.data(), V, sp, seed_for(sp, (int)history.size()));
                    history.push_back(next);
                    emit(next);
                    pending = next;
                    if (is_stop(next)) break;
                    continue;
                }

                // DraftRuntime::generate_draft_tokens (src/draft_runtime.cpp:46-95).
                std::vector<uint32_t> drafts;
                std::vector<std::vector<float>> draft_logits;
                {
                    if (consumed > history.size()) consumed = 0;
                    drf.truncate(history, (uint32_t)consumed);
                    while (consumed + 1 < history.size()) {
                        drf.forward(history[consumed], (uint32_t)consumed);
                        ++consumed;
                    }
                    uint32_t cur = history.back();
                    uint32_t pos = (uint32_t)consumed;
                    for (uint32_t step = 0; step + 1 < K; ++step) {
                        auto l = drf.forward(cur, pos);
                        ++pos;
                        const uint64_t ss = splitmix64(sp.has_seed ? (sp.seed + step) : (1337 + step));
                        const uint32_t cand = sample_token(l.data(), V, sp, ss);
                        drafts.push_back(cand);
                        draft_logits.push_back(std::move(l));
                        cur = cand;
                    }
                    consumed = history.size();
                }

                // Verify pass: [pending, d1..d_{K-1}] at positions history.size()-1 onward.
                const uint32_t base = (uint32_t)(history.size() - 1);
                std::vector<std::vector<float>> verify;
                verify.push_back(tgt.forward(pending, base));
                for (uint32_t i = 0; i < drafts.size(); ++i) verify.push_back(tgt.forward(drafts[i], base + 1 + i));
                std::vector<const float*> per_pos;
                for (auto& v : verify) per_pos.push_back(v.data());

                auto ev = spec.evaluate_verification(drafts, per_pos, V, sp,
                                                     seed_for(sp, (int)history.size()), draft_logits);
                int this_emit = 0;
                bool stop = false;
                for (uint32_t t : ev.accepted_tokens) {
                    if (emitted >= max_tokens) { stop = true; break; }
                    history.push_back(t);
                    emit(t);
                    ++this_emit;
                    pending = t;
                    if (is_stop(t)) { stop = true; break; }
                }
                // Target: positions beyond the kept history (minus the pending token, which is
                // forwarded next round) are rejected drafts.
                tgt.truncate(history, (uint32_t)(history.size() - 1));
                // DraftRuntime::accept, capped at what the drafter forwarded (see header).
                consumed = std::min<size_t>(history.size() - 1, drf.fed);

                if (rounds < max_rounds) {
                    round_info[3 * rounds + 0] = (int)drafts.size();
                    round_info[3 * rounds + 1] = (int)ev.num_accepted;
                    round_info[3 * rounds + 2] = this_emit;
                }
                ++rounds;
                drafted_total += (uint32_t)drafts.size();
                accepted_total += ev.num_accepted;
                if (drafting && gate_window >= 0 && drafted_total >= (uint32_t)gate_window &&
                    (double)accepted_total / drafted_total < gate_min_accept) {
                    drafting = false;
                }
                if (stop) break;
            }
            *n_rounds = rounds;
            return emitted;
        }

        // Non-speculative loop (src/runner.cpp:2314-2344).
        for (int step = 0; step < max_tokens; ++step) {
            const uint32_t pos = (uint32_t)(history.size() - 1);
            const uint32_t next = sample_token(logits.data(), V, sp, seed_for(sp, (int)pos));
            history.push_back(next);
            emit(next);
            if (is_stop(next)) break;
            if (emitted >= max_tokens) break;
            logits = tgt.forward(next, (uint32_t)(history.size() - 1));
        }
        *n_rounds = 0;
        return emitted;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

}  // extern "C"

// ---- tokenizer ---------------------------------------------------------------------------

namespace {
struct RefTok {
    Tokenizer tok;
    std::string out;
};
struct RefDetok {
    RefDetok(const Tokenizer& t, bool skip) : d(t, skip) {}
    IncrementalDetokenizer d;
    std::string out;
};
struct RefStop {
    StreamingStopMatcher m;
    std::string out;
};
const char* hand_out(std::string& buf, std::string s, size_t* out_len) {
    buf = std::move(s);
    if (out_len) *out_len = buf.size();
    return buf.c_str();
}
}  // namespace

extern "C" {

// Tokenizer::load_vocabulary(path) then set_architecture(arch) (0 Gemma-4, 1 Muse-Glimmer);
// a null path leaves the tokenizer empty (its default-constructed state).
void* ref_tok_open(const char* path, int arch) {
    try {
        auto t = std::make_unique<RefTok>();
        if (path) t->tok.load_vocabulary(path);
        t->tok.set_architecture(arch == 1 ? ModelArch::MUSE_GLIMMER : ModelArch::GEMMA4);
        return t.release();
    } catch (const std::exception& e) {
        g_err = e.what();
        return nullptr;
    }
}
void ref_tok_close(void* h) { delete static_cast<RefTok*>(h); }

int ref_tok_encode(void* h, const char* text, size_t len, int add_bos, uint32_t* out, int cap) {
    try {
        const auto ids = static_cast<RefTok*>(h)->tok.encode(std::string(text, len), add_bos != 0);
        for (size_t i = 0; i < ids.size() && (int)i < cap; ++i) out[i] = ids[i];
        return (int)ids.size();
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

const char* ref_tok_decode(void* h, const uint32_t* ids, int n, int skip_special, size_t* out_len) {
    try {
        auto* t = static_cast<RefTok*>(h);
        return hand_out(t->out, t->tok.decode(std::vector<uint32_t>(ids, ids + n), skip_special != 0), out_len);
    } catch (const std::exception& e) {
        g_err = e.what();
        return nullptr;
    }
}

const char* ref_tok_decode_single(void* h, uint32_t id, int skip_special, size_t* out_len) {
    auto* t = static_cast<RefTok*>(h);
    return hand_out(t->out, t->tok.decode_single(id, skip_special != 0), out_len);
}

// apply_chat_template over n (role, content) pairs.
const char* ref_tok_chat_template(void* h, const char* const* roles, const char* const* contents, int n) {
    try {
        auto* t = static_cast<RefTok*>(h);
        std::vector<Tokenizer::ChatMessage> msgs;
        for (int i = 0; i < n; ++i) msgs.push_back({roles[i], contents[i]});
        return hand_out(t->out, t->tok.apply_chat_template(msgs), nullptr);
    } catch (const std::exception& e) {
        g_err = e.what();
        return nullptr;
    }
}

// out[0..6) = bos, eos, pad, unk, end_of_turn, vocab_size; out[6] = loaded.
void ref_tok_special_ids(void* h, uint32_t* out7) {
    const Tokenizer& t = static_cast<RefTok*>(h)->tok;
    const uint32_t v[7] = {t.bos_id(), t.eos_id(), t.pad_id(), t.unk_id(), t.end_of_turn_id(), t.vocab_size(),
                           t.is_loaded() ? 1u : 0u};
    std::memcpy(out7, v, sizeof(v));
}

int ref_tok_stop_ids(void* h, uint32_t* out, int cap) {
    const auto& s = static_cast<RefTok*>(h)->tok.stop_token_ids();
    for (size_t i = 0; i < s.size() && (int)i < cap; ++i) out[i] = s[i];
    return (int)s.size();
}

int ref_tok_byte_value(void* h, uint32_t id, uint8_t* value) {
    return static_cast<RefTok*>(h)->tok.is_byte_fallback(id, *value) ? 1 : 0;
}

int ref_tok_is_special(void* h, uint32_t id) { return static_cast<RefTok*>(h)->tok.is_special_token(id) ? 1 : 0; }

void* ref_detok_create(void* h, int skip_special) {
    return new RefDetok(static_cast<RefTok*>(h)->tok, skip_special != 0);
}
const char* ref_detok_push(void* d, uint32_t id, size_t* out_len) {
    auto* x = static_cast<RefDetok*>(d);
    return hand_out(x->out, x->d.push(id), out_len);
}
const char* ref_detok_finish(void* d, size_t* out_len) {
    auto* x = static_cast<RefDetok*>(d);
    return hand_out(x->out, x->d.finish(), out_len);
}
void ref_detok_destroy(void* d) { delete static_cast<RefDetok*>(d); }

void* ref_stop_create(const char* const* stops, int n) {
    std::vector<std::string> v;
    for (int i = 0; i < n; ++i) v.emplace_back(stops[i]);
    auto* m = new RefStop;
    m->m = StreamingStopMatcher(std::move(v));
    return m;
}
const char* ref_stop_push(void* m, const char* text, size_t len, size_t* out_len) {
    auto* x = static_cast<RefStop*>(m);
    return hand_out(x->out, x->m.push(std::string_view(text, len)), out_len);
}
const char* ref_stop_finish(void* m, size_t* out_len) {
    auto* x = static_cast<RefStop*>(m);
    return hand_out(x->out, x->m.finish(), out_len);
}
int ref_stop_stopped(void* m, const char** matched) {
    auto* x = static_cast<RefStop*>(m);
    if (matched) *matched = x->m.matched().c_str();
    return x->m.stopped() ? 1 : 0;
}
void ref_stop_destroy(void* m) { delete static_cast<RefStop*>(m); }

const char* ref_utf8_repair(const char* in, size_t len, int flush_all, size_t* consumed, size_t* out_len) {
    thread_local std::string buf;
    std::string out;
    const size_t used = utf8_repair(std::string_view(in, len), flush_all != 0, out);
    if (consumed) *consumed = used;
    return hand_out(buf, std::move(out), out_len);
}

}  // extern "C"
