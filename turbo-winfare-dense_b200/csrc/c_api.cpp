// The engine's C ABI (include/g4dense/c_api.h). Exceptions never cross it: failures return
// nullptr / -1 with a thread-local message, as src/c_api.cpp does.
#include "g4dense/c_api.h"

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <memory>
#include <sstream>
#include <string>
#include <vector>

#include "format.h"
#include "runner.h"
#include "tokenizer.h"

#ifdef G4B_HAVE_NCCL
#include <nccl.h>
#endif

namespace {

thread_local std::string g_last_error;
void set_error(const std::string& m) { g_last_error = m; }
void clear_error() { g_last_error.clear(); }

// A tokenizer behind the C ABI, with the buffer its returned strings live in.
struct TokHandle {
    g4b::Tokenizer tok;
    bool engine_owned{false};  // the engine's own tokenizer: g4dense_tokenizer_destroy ignores it
    std::string out;
};
struct DetokHandle {
    explicit DetokHandle(const g4b::Tokenizer& t, bool skip) : d(t, skip) {}
    g4b::IncrementalDetokenizer d;
    std::string out;
};
struct StopHandle {
    g4b::StreamingStopMatcher m;
    std::string out;
};

const char* give(std::string& buf, std::string s, size_t* out_len) {
    buf = std::move(s);
    if (out_len) *out_len = buf.size();
    return buf.c_str();
}

// Runs `body` so that no exception (an allocation failure included) crosses the C ABI: on one,
// the message goes to the thread's last error and `failed` is returned.
template <class R, class F>
R guarded(R failed, F&& body) {
    try {
        return body();
    } catch (const std::exception& e) {
        set_error(e.what());
    } catch (...) {
        set_error("unknown C++ exception");
    }
    return failed;
}

struct EngineHandle {
    std::unique_ptr<g4b::Engine> engine;
    std::unique_ptr<TokHandle> tok;  // null: the text entry points fail
    std::atomic<bool> cancel{false};
    std::string last_response, last_telemetry;
    std::vector<uint32_t> last_tokens;
    int last_stop_reason{0};
    int draft_k{0};
    int64_t stop_token{-1};
    std::vector<uint32_t> replay;
    double mismatch_rate{0};
    uint64_t mismatch_seed{0};
    bool device_sampling{true};
    double gate_min_accept{0.45};
    int gate_window{24};
    void* nccl_comm{nullptr};
    ~EngineHandle() {
        engine.reset();
#ifdef G4B_HAVE_NCCL
        if (nccl_comm) ncclCommDestroy((ncclComm_t)nccl_comm);
#endif
    }
};

// MTP drafter geometries: the 31B's assistant (tools/convert_hf_assistant.py:49-66 defaults) and
// "mtp-small", a 4-layer drafter sized for tests, with attention geometry taken from `t`.
bool mtp_preset_header(const std::string& name, const g4b::G4DenseHeader& t, g4b::G4MtpHeader& m) {
    std::memset(&m, 0, sizeof(m));
    m.num_layers = 4;
    m.backbone_hidden_size = t.d_model;
    m.vocab_size = t.vocab_size;
    m.num_kv_heads = t.num_kv_heads;
    m.head_dim = t.head_dim;
    m.global_head_dim = t.global_head_dim ? t.global_head_dim : 512;
    m.global_kv_heads = t.global_kv_heads ? t.global_kv_heads : 4;
    m.sliding_window = t.sliding_window;
    m.global_layer_mask = 1ull << 3;  // sliding x3, then full attention
    if (name == "gemma4-31b-assistant") {
        m.hidden_size = 1024;
        m.intermediate_size = 8192;
        m.num_q_heads = 32;
    } else if (name == "mtp-small") {
        m.hidden_size = 128;
        m.intermediate_size = 512;
        m.num_q_heads = t.num_q_heads;
    } else {
        return false;
    }
    return true;
}

// Model geometries for device-generated weights, with optional ":layers=N" and ":shard=S"
// overrides (comma-separated). shard=S gives the geometry one rank of an S-way tensor-parallel
// run holds (query and KV heads, FFN width and vocabulary divided by S, at least one KV head), so
// a single GPU can time one shard's kernels without the peer exchange.
bool preset_header(const std::string& spec, g4b::G4DenseHeader& h) {
    std::string name = spec;
    int layers = -1, shard = 1;
    const size_t colon = spec.find(':');
    if (colon != std::string::npos) {
        name = spec.substr(0, colon);
        std::string rest = spec.substr(colon + 1);
        while (!rest.empty()) {
            const size_t comma = rest.find(',');
            const std::string kv = rest.substr(0, comma);
            if (kv.rfind("layers=", 0) == 0) layers = std::atoi(kv.c_str() + 7);
            else if (kv.rfind("shard=", 0) == 0) shard = std::atoi(kv.c_str() + 6);
            else return false;
            rest = comma == std::string::npos ? std::string() : rest.substr(comma + 1);
        }
        if (shard < 1) return false;
    }
    std::memset(&h, 0, sizeof(h));
    h.rope_theta_local = 10000.0f;
    h.rope_theta_global = 1000000.0f;
    h.rope_scaling = 1.0f;
    h.final_logit_softcapping = 30.0f;
    h.scale_dtype = 1;
    if (name == "gemma4-31b") {
        // docs/FORWARD_PASS.md constants: global layers every 6th from layer 5.
        h.num_layers = 60; h.d_model = 5376; h.d_ff = 21504; h.num_q_heads = 32; h.num_kv_heads = 16;
        h.head_dim = 256; h.vocab_size = 262144; h.sliding_window = 1024;
        h.global_layer_mask = 0x0820820820820820ull; h.global_head_dim = 512; h.global_kv_heads = 4;
    } else if (name == "gemma4-e2b") {
        h.num_layers = 35; h.d_model = 1536; h.d_ff = 6144; h.num_q_heads = 8; h.num_kv_heads = 1;
        h.head_dim = 256; h.vocab_size = 262144; h.sliding_window = 512;
    } else if (name == "config0-target") {
        h.num_layers = 4; h.d_model = 256; h.d_ff = 1024; h.num_q_heads = 4; h.num_kv_heads = 1;
        h.head_dim = 64; h.vocab_size = 4096; h.sliding_window = 1024;
    } else if (name == "config0-draft") {
        h.num_layers = 2; h.d_model = 128; h.d_ff = 512; h.num_q_heads = 2; h.num_kv_heads = 1;
        h.head_dim = 64; h.vocab_size = 4096; h.sliding_window = 1024;
    } else {
        return false;
    }
    if (layers > 0 && layers <= 60) {
        h.num_layers = (uint32_t)layers;
        h.global_layer_mask &= (layers == 64) ? ~0ull : ((1ull << layers) - 1);
    }
    if (shard > 1) {
        if (h.num_q_heads % shard || h.d_ff % (64 * shard) || h.vocab_size % shard) return false;
        h.num_q_heads /= shard;
        h.num_kv_heads = std::max(1u, h.num_kv_heads / shard);
        if (h.global_kv_heads) h.global_kv_heads = std::max(1u, h.global_kv_heads / shard);
        h.d_ff /= shard;
        h.vocab_size /= shard;
    }
    for (uint32_t l = 0; l < h.num_layers; ++l) h.layer_d_ff[l] = h.d_ff;
    return true;
}

g4b::GenerationOptions to_gen(const EngineHandle* e, const G4DenseGenerationOptions* o) {
    g4b::GenerationOptions g;
    if (o) {
        g.max_tokens = o->max_tokens;
        g.sampling.temperature = o->temperature;
        g.sampling.top_p = o->top_p;
        g.sampling.top_k = o->top_k;
        g.sampling.repetition_penalty = o->repetition_penalty;
        g.sampling.has_seed = o->has_seed != 0;
        g.sampling.seed = o->seed;
    }
    g.speculative_enabled = e->draft_k > 0 && e->engine->has_drafter();
    g.draft_k = (uint32_t)std::max(0, e->draft_k);
    g.stop_token = e->stop_token;
    g.replay = e->replay;
    g.mismatch_rate = e->mismatch_rate;
    g.mismatch_seed = e->mismatch_seed;
    g.device_sampling = e->device_sampling;
    g.gate_min_accept = e->gate_min_accept;
    g.gate_window = e->gate_window;
    return g;
}

// Where the engine's tokenizer comes from: the config, $G4DENSE_TOKENIZER, tokenizer.json beside
// the container, then tokenizer.json in the working directory (the first place the reference's
// resolve_resource_path looks, src/manifest.cpp:200-212). "" when none is found.
std::string tokenizer_file(const G4DenseEngineConfig* cfg) {
    if (cfg->tokenizer_path && *cfg->tokenizer_path) return cfg->tokenizer_path;
    if (const char* env = std::getenv("G4DENSE_TOKENIZER"); env && *env) return env;
    namespace fs = std::filesystem;
    std::error_code ec;
    if (cfg->container_path && *cfg->container_path) {
        const fs::path beside = fs::path(cfg->container_path).parent_path() / "tokenizer.json";
        if (fs::is_regular_file(beside, ec)) return beside.string();
    }
    if (fs::is_regular_file("tokenizer.json", ec)) return "tokenizer.json";
    return "";
}

// ForwardRunner::generate(prompt, options) (src/runner.cpp:2060-2347): chat template or raw
// encode, then the engine's decode loop, stopping after a tokenizer stop id; every emitted token
// reaches on_token with its decode_single piece, and the pieces are returned concatenated.
const char* generate_text(EngineHandle* e, const std::string& prompt, bool chat, const G4DenseGenerationOptions* o,
                          G4DenseTokenCallback on_token, void* user) {
    if (!e->tok) throw std::runtime_error("ForwardRunner::generate: Tokenizer is not loaded or missing");
    const g4b::Tokenizer& tk = e->tok->tok;
    // The template emits the literal "<bos>", so the templated text is encoded without another.
    const std::vector<uint32_t> ids =
        chat ? tk.encode(tk.chat_template({{"user", prompt}}), false) : tk.encode(prompt, true);
    if (ids.empty()) throw std::runtime_error("ForwardRunner::generate: prompt encoded to empty token sequence");
    g4b::GenerationOptions g = to_gen(e, o);
    g.stop_tokens = tk.stop_ids();
    e->cancel.store(false);
    e->last_response.clear();
    int idx = 0;
    auto cb = [&](uint32_t t) {
        const std::string piece = tk.decode_single(t);
        e->last_response += piece;
        return on_token ? on_token(user, idx++, t, piece.c_str()) != 0 : true;
    };
    e->last_tokens = e->engine->generate(ids, g, cb, &e->cancel);
    e->last_stop_reason = e->engine->last_stats().stop_reason;
    return e->last_response.c_str();
}

}  // namespace

extern "C" {

G4DENSE_API const char* g4dense_engine_last_error(void) { return g_last_error.c_str(); }

G4DENSE_API void g4dense_options_default(G4DenseGenerationOptions* out) {
    if (!out) return;
    out->max_tokens = 512;
    out->temperature = 0.2f;
    out->top_p = 0.95f;
    out->top_k = 64;
    out->repetition_penalty = 1.0f;
    out->has_seed = 0;
    out->seed = 0;
    out->system_prompt = nullptr;
    out->stop_strings = nullptr;
    out->stop_count = 0;
    out->tier_id = 1;
}

G4DENSE_API void g4dense_config_default(G4DenseEngineConfig* c) {
    if (!c) return;
    std::memset(c, 0, sizeof(*c));
    c->max_context = 4096;
    c->tp_size = 1;
    c->device = -1;
    c->gate_min_accept = 0.45;
    c->gate_window = 24;
}

G4DENSE_API int g4dense_nccl_unique_id(void* out128) {
    clear_error();
    if (!out128) {
        set_error("Null output buffer");
        return -1;
    }
#ifdef G4B_HAVE_NCCL
    ncclUniqueId id;
    if (ncclGetUniqueId(&id) != ncclSuccess) {
        set_error("ncclGetUniqueId failed");
        return -1;
    }
    std::memcpy(out128, &id, sizeof(id));
    return 0;
#else
    (void)out128;
    set_error("built without NCCL");
    return -1;
#endif
}

G4DENSE_API void* g4dense_engine_create_ex(const G4DenseEngineConfig* cfg) {
    clear_error();
    if (!cfg) {
        set_error("null config");
        return nullptr;
    }
    try {
        if (cfg->device >= 0) g4b::cuda_check(cudaSetDevice(cfg->device), "cudaSetDevice");
        int ndev = 0;
        g4b::cuda_check(cudaGetDeviceCount(&ndev), "cudaGetDeviceCount");
        auto h = std::make_unique<EngineHandle>();
        g4b::ModelOptions mo;
        mo.max_context = cfg->max_context > 0 ? cfg->max_context : 4096;
        mo.kv_bf16 = cfg->kv_bf16;
        mo.rank = cfg->tp_rank;
        mo.tp = cfg->tp_size > 0 ? cfg->tp_size : 1;
        if (const char* g = std::getenv("G4DENSE_NO_GRAPHS")) mo.use_graphs = std::atoi(g) == 0;
        if (mo.tp > 1) {
#ifdef G4B_HAVE_NCCL
            if (!cfg->nccl_unique_id) throw std::invalid_argument("tensor parallelism needs an NCCL unique id");
            ncclUniqueId id;
            std::memcpy(&id, cfg->nccl_unique_id, sizeof(id));
            ncclComm_t comm;
            if (ncclCommInitRank(&comm, mo.tp, id, mo.rank) != ncclSuccess)
                throw std::runtime_error("ncclCommInitRank failed");
            h->nccl_comm = comm;
            mo.nccl_comm = comm;
#else
            throw std::invalid_argument("built without NCCL");
#endif
        }
        auto target = std::make_unique<g4b::DeviceModel>(mo);
        if (cfg->container_path && *cfg->container_path) {
            target->load_container(cfg->container_path);
        } else if (cfg->synthetic_preset) {
            g4b::G4DenseHeader gh;
            if (!preset_header(cfg->synthetic_preset, gh)) throw std::invalid_argument("unknown synthetic preset");
            target->load_synthetic(gh, cfg->synthetic_seed, cfg->synthetic_centered != 0);
        } else {
            throw std::invalid_argument("no target container or synthetic preset");
        }
        const cudaStream_t st = target->stream();
        h->engine = std::make_unique<g4b::Engine>(std::move(target));
        bool mtp = false;
        if (cfg->draft_path && *cfg->draft_path) {
            if (FILE* f = std::fopen(cfg->draft_path, "rb")) {
                uint32_t magic = 0;
                if (std::fread(&magic, 4, 1, f) == 1) mtp = magic == g4b::G4MtpHeader::kMagic;
                std::fclose(f);
            }
        } else if (cfg->draft_preset) {
            mtp = std::strncmp(cfg->draft_preset, "mtp-", 4) == 0 ||
                  std::strcmp(cfg->draft_preset, "gemma4-31b-assistant") == 0;
        }
        if (mtp) {
            // The MTP assistant drafter (src/mtp_runner.cpp) reads the target's KV rings, embedding
            // and final hidden states, so it shares the target's device and stream.
            if (mo.tp != 1) throw std::invalid_argument("the MTP drafter runs without tensor parallelism");
            g4b::DeviceModel& T = h->engine->target();
            T.enable_hidden_out();
            g4b::ModelOptions dopt;
            dopt.max_context = mo.max_context;
            dopt.kv_bf16 = mo.kv_bf16;
            dopt.use_graphs = mo.use_graphs;
            dopt.prefill_tc = false;
            dopt.stream = st;
            auto d = std::make_unique<g4b::DeviceModel>(dopt);
            if (cfg->draft_path && *cfg->draft_path) {
                d->load_mtp(cfg->draft_path, T);
            } else {
                g4b::G4MtpHeader mh;
                if (!mtp_preset_header(cfg->draft_preset, T.header(), mh))
                    throw std::invalid_argument("unknown MTP drafter preset");
                d->load_mtp_synthetic(mh, cfg->draft_seed, cfg->synthetic_centered != 0, T);
            }
            h->engine->set_mtp(std::move(d));
        } else if (((cfg->draft_path && *cfg->draft_path) || cfg->draft_preset) && mo.rank != 0) {
            // Tensor parallelism: the drafter runs on rank 0 alone; this rank receives each
            // round's drafts by broadcast.
            h->engine->set_remote_draft(true);
        } else if ((cfg->draft_path && *cfg->draft_path) || cfg->draft_preset) {
            // The drafter runs whole on one GPU (rank 0 under tensor parallelism) on its own
            // stream, so its prompt catch-up overlaps the target's prefill; the engine orders the
            // two streams with events where a round's passes depend on each other.
            g4b::ModelOptions dopt;
            dopt.max_context = mo.max_context;
            dopt.kv_bf16 = mo.kv_bf16;
            dopt.use_graphs = mo.use_graphs;
            auto d = std::make_unique<g4b::DeviceModel>(dopt);
            if (cfg->draft_path && *cfg->draft_path) {
                d->load_container(cfg->draft_path);
            } else {
                g4b::G4DenseHeader dh;
                if (!preset_header(cfg->draft_preset, dh)) throw std::invalid_argument("unknown drafter preset");
                d->load_synthetic(dh, cfg->draft_seed, cfg->synthetic_centered != 0);
            }
            h->engine->set_draft(std::move(d));
        }
        h->draft_k = cfg->draft_k;
        h->gate_min_accept = cfg->gate_min_accept;
        h->gate_window = cfg->gate_window;
        // The runner sets the tokenizer's architecture from the container header
        // (src/runner.cpp:265), which decides the chat template and the stop ids.
        if (const std::string tp = tokenizer_file(cfg); !tp.empty()) {
            auto t = std::make_unique<TokHandle>();
            t->engine_owned = true;
            t->tok.load(tp);
            t->tok.set_arch(h->engine->target().header().arch_type == 1 ? g4b::Tokenizer::Arch::MuseGlimmer
                                                                         : g4b::Tokenizer::Arch::Gemma4);
            h->tok = std::move(t);
        }
        return h.release();
    } catch (const std::exception& e) {
        set_error(e.what());
        return nullptr;
    }
}

G4DENSE_API void* g4dense_engine_create(const char* container_path) {
    clear_error();
    G4DenseEngineConfig c;
    g4dense_config_default(&c);
    // The default name is a literal, so no allocation is needed for the path.
    c.container_path = (container_path && *container_path) ? container_path : "gemma-4-31b-dense.g4dense";
    // Speculation is opt-in, as in the reference; these environment variables enable it
    // without changing the signature.
    if (const char* d = std::getenv("G4DENSE_DRAFT_MODEL")) c.draft_path = d;
    if (const char* k = std::getenv("G4DENSE_SPEC_K")) c.draft_k = std::atoi(k);
    if (const char* m = std::getenv("G4DENSE_SPEC_GATE_MIN_ACCEPT")) c.gate_min_accept = std::atof(m);
    if (const char* w = std::getenv("G4DENSE_SPEC_GATE_WINDOW")) c.gate_window = std::max(0, std::atoi(w));
    return g4dense_engine_create_ex(&c);
}

G4DENSE_API void g4dense_engine_destroy(void* handle) { delete static_cast<EngineHandle*>(handle); }

G4DENSE_API const char* g4dense_engine_generate(void* handle, const char* prompt, int max_tokens) {
    clear_error();
    if (!handle || !prompt) {
        set_error("Invalid handle or null prompt");
        return nullptr;
    }
    try {
        G4DenseGenerationOptions o;
        g4dense_options_default(&o);  // temperature 0.2, top_p 0.95, top_k 64 (src/c_api.cpp:93-96)
        o.max_tokens = max_tokens > 0 ? max_tokens : 512;
        return generate_text(static_cast<EngineHandle*>(handle), prompt, true, &o, nullptr, nullptr);
    } catch (const std::exception& ex) {
        set_error(ex.what());
        return nullptr;
    }
}

G4DENSE_API const char* g4dense_engine_generate_ex(void* handle, const char* messages_json,
                                                   const G4DenseGenerationOptions* opts, G4DenseTokenCallback on_token,
                                                   void* user) {
    clear_error();
    if (!handle || !messages_json) {
        set_error("Invalid handle or null messages");
        return nullptr;
    }
    try {
        return generate_text(static_cast<EngineHandle*>(handle), messages_json, true, opts, on_token, user);
    } catch (const std::exception& ex) {
        set_error(ex.what());
        return nullptr;
    }
}

G4DENSE_API const char* g4dense_engine_generate_text(void* handle, const char* prompt, int use_chat_template,
                                                     const G4DenseGenerationOptions* opts,
                                                     G4DenseTokenCallback on_token, void* user) {
    clear_error();
    if (!handle || !prompt) {
        set_error("Invalid handle or null prompt");
        return nullptr;
    }
    try {
        return generate_text(static_cast<EngineHandle*>(handle), prompt, use_chat_template != 0, opts, on_token,
                             user);
    } catch (const std::exception& ex) {
        set_error(ex.what());
        return nullptr;
    }
}

G4DENSE_API const char* g4dense_engine_generate_tokens(void* handle, const unsigned int* prompt_ids, int n_prompt,
                                                       const G4DenseGenerationOptions* opts,
                                                       G4DenseTokenCallback on_token, void* user) {
    clear_error();
    if (!handle || !prompt_ids || n_prompt <= 0) {
        set_error("Invalid handle or empty prompt");
        return nullptr;
    }
    auto* e = static_cast<EngineHandle*>(handle);
    try {
        e->cancel.store(false);
        const g4b::GenerationOptions g = to_gen(e, opts);
        std::vector<uint32_t> prompt(prompt_ids, prompt_ids + n_prompt);
        int idx = 0;
        auto cb = [&](uint32_t t) {
            if (!on_token) return true;
            return on_token(user, idx++, t, "") != 0;
        };
        e->last_tokens = e->engine->generate(prompt, g, cb, &e->cancel);
        const g4b::GenStats& s = e->engine->last_stats();
        e->last_stop_reason = s.stop_reason;
        std::ostringstream ss;
        ss << "{\"tokens\": " << e->last_tokens.size() << ", \"drafted\": " << s.drafted << ", \"accepted\": "
           << s.accepted << ", \"rounds\": " << s.rounds << ", \"ttft_ms\": " << s.ttft_ms << ", \"total_ms\": "
           << s.total_ms << "}";
        e->last_response = ss.str();
        return e->last_response.c_str();
    } catch (const std::exception& ex) {
        set_error(ex.what());
        return nullptr;
    }
}

G4DENSE_API int g4dense_engine_last_tokens(void* handle, unsigned int* out, int cap) {
    if (!handle || !out || cap < 0) return 0;
    auto* e = static_cast<EngineHandle*>(handle);
    const int n = std::min<int>(cap, (int)e->last_tokens.size());
    std::memcpy(out, e->last_tokens.data(), (size_t)n * sizeof(unsigned int));
    return n;
}

G4DENSE_API int g4dense_engine_last_rounds(void* handle, int* out, int cap_triples) {
    if (!handle || !out || cap_triples < 0) return 0;
    auto* e = static_cast<EngineHandle*>(handle);
    const auto& ri = e->engine->last_stats().round_info;
    const int n = std::min<int>(cap_triples, (int)ri.size() / 3);
    std::memcpy(out, ri.data(), (size_t)n * 3 * sizeof(int));
    return n;
}

G4DENSE_API int g4dense_engine_forward_batch(void* handle, const unsigned int* token_ids, int batch, int base_position,
                                             float* out_logits, int all_positions) {
    clear_error();
    if (!handle || !token_ids || batch <= 0 || base_position < 0) {
        set_error("Invalid arguments");
        return -1;
    }
    try {
        static_cast<EngineHandle*>(handle)->engine->forward_batch(token_ids, (uint32_t)batch, (uint32_t)base_position,
                                                                  out_logits, all_positions != 0);
        return 0;
    } catch (const std::exception& e) {
        set_error(e.what());
        return -1;
    }
}

// Greedy drafting by the separate drafter model, DraftRuntime::generate_draft_tokens's greedy case
// (src/draft_runtime.cpp:46-95) on the device: k chained one-row steps from `token` at position
// `pos` over the drafter's current KV cache, each step's argmax feeding the next. Writes the k
// drafted tokens and, when out_logits is non-null, each step's softcapped logits [k][vocab].
G4DENSE_API int g4dense_engine_draft_steps(void* handle, unsigned int token, int pos, int k, unsigned int* out_tokens,
                                           float* out_logits) {
    clear_error();
    if (!handle || pos < 0 || k < 1 || k > 64 || !out_tokens) {
        set_error("Invalid arguments");
        return -1;
    }
    try {
        g4b::Engine& E = *static_cast<EngineHandle*>(handle)->engine;
        if (!E.draft()) throw std::invalid_argument("no drafter model loaded");
        g4b::DeviceModel& m = E.draft()->model();
        if (pos + k > m.max_context()) throw std::invalid_argument("pos + k exceeds the drafter's KV capacity");
        const int V = (int)m.header().vocab_size;
        g4b::StepParams p{};
        p.base_pos = pos;
        p.tokens[0] = token % (unsigned)V;
        m.push_params(1, p, 1);
        for (int s = 0; s < k; ++s) {
            m.enqueue(1, g4b::PassKind::DraftStep, out_logits != nullptr, m.chain_dev());
            if (out_logits)
                g4b::cuda_check(cudaMemcpyAsync(out_logits + (size_t)s * V, m.logits_dev(), (size_t)V * 4,
                                                cudaMemcpyDeviceToHost, m.stream()),
                                "logits");
        }
        g4b::cuda_check(cudaMemcpyAsync(out_tokens, m.chain_dev(), (size_t)k * 4, cudaMemcpyDeviceToHost, m.stream()),
                        "tokens");
        g4b::cuda_check(cudaStreamSynchronize(m.stream()), "sync");
        m.check_device_error();
        return 0;
    } catch (const std::exception& ex) {
        set_error(ex.what());
        return -1;
    }
}

G4DENSE_API int g4dense_engine_mtp_draft(void* handle, unsigned int seed_token, int context_length, int hidden_row,
                                         int k, unsigned int* out_tokens, float* out_logits) {
    clear_error();
    if (!handle || context_length < 2 || hidden_row < 0 || k < 1 || !out_tokens) {
        set_error("Invalid arguments");
        return -1;
    }
    try {
        g4b::Engine& E = *static_cast<EngineHandle*>(handle)->engine;
        g4b::DeviceModel* Mt = E.mtp();
        if (!Mt) throw std::invalid_argument("no MTP drafter loaded");
        if (hidden_row >= E.target().max_rows()) throw std::invalid_argument("hidden_row out of range");
        const int V = (int)Mt->header().vocab_size;
        uint32_t tok = seed_token;
        for (int s = 0; s < k; ++s) {
            g4b::StepParams p{};
            p.base_pos = context_length - 2;
            p.tokens[0] = tok;
            p.aux = hidden_row;
            Mt->push_params(1, p, 1);
            Mt->enqueue(1, s == 0 ? g4b::PassKind::MtpFirst : g4b::PassKind::MtpNext, out_logits != nullptr, nullptr);
            const HeadResult r = Mt->fetch_result();
            tok = r.argmax[0];
            out_tokens[s] = tok;
            if (out_logits)
                g4b::cuda_check(cudaMemcpy(out_logits + (size_t)s * V, Mt->logits_dev(), (size_t)V * 4,
                                           cudaMemcpyDeviceToHost),
                                "logits");
        }
        Mt->check_device_error();
        return 0;
    } catch (const std::exception& e) {
        set_error(e.what());
        return -1;
    }
}

G4DENSE_API int g4dense_engine_set_decode_options(void* handle, long long stop_token, int draft_k,
                                                  const unsigned int* replay, int replay_len, double mismatch_rate,
                                                  unsigned long long mismatch_seed) {
    clear_error();
    if (!handle || replay_len < 0 || mismatch_rate < 0 || mismatch_rate > 1) {
        set_error("Invalid arguments");
        return -1;
    }
    auto* e = static_cast<EngineHandle*>(handle);
    return guarded(-1, [&] {
        e->replay.assign(replay, replay ? replay + replay_len : replay);
        e->stop_token = stop_token;
        if (draft_k >= 0) e->draft_k = draft_k;
        e->mismatch_rate = mismatch_rate;
        e->mismatch_seed = mismatch_seed;
        return 0;
    });
}

G4DENSE_API int g4dense_engine_set_device_sampling(void* handle, int on) {
    clear_error();
    if (!handle) {
        set_error("Invalid arguments");
        return -1;
    }
    static_cast<EngineHandle*>(handle)->device_sampling = on != 0;
    return 0;
}

G4DENSE_API const char* g4dense_engine_get_telemetry(void* handle) {
    if (!handle) return "{}";
    auto* e = static_cast<EngineHandle*>(handle);
    try {
        e->last_telemetry = e->engine->telemetry_json();
    } catch (const std::exception& ex) {
        e->last_telemetry = "{}";
    }
    return e->last_telemetry.c_str();
}

G4DENSE_API int g4dense_engine_last_stop_reason(void* handle) {
    if (!handle) return 0;
    return static_cast<EngineHandle*>(handle)->last_stop_reason;
}

G4DENSE_API int g4dense_engine_switch_tier(void* handle, int tier_id) {
    clear_error();
    if (!handle) {
        set_error("Null handle");
        return -1;
    }
    if (tier_id < 0) {
        set_error("Invalid tier id");
        return -1;
    }
    return 0;
}

G4DENSE_API int g4dense_engine_last_stats(void* handle, double* out, int n) {
    if (!handle || !out) return 0;
    const g4b::GenStats& s = static_cast<EngineHandle*>(handle)->engine->last_stats();
    const double v[] = {(double)s.emitted, s.decode_gpu_ms, s.ttft_ms, s.total_ms, (double)s.drafted,
                        (double)s.accepted, (double)s.rounds, (double)s.gated_steps, (double)s.launches,
                        (double)s.h2d_bytes, (double)s.d2h_bytes, s.decode_ms};
    const int m = std::min<int>(n, (int)(sizeof(v) / sizeof(v[0])));
    for (int i = 0; i < m; ++i) out[i] = v[i];
    return m;
}

G4DENSE_API double g4dense_engine_profile_gemms(void* handle, int batch, int reps, unsigned long long* bytes,
                                                int* launches) {
    clear_error();
    if (!handle || batch < 1 || batch > 16 || reps < 1) {
        set_error("Invalid arguments");
        return -1.0;
    }
    try {
        uint64_t b = 0;
        const double ms = static_cast<EngineHandle*>(handle)->engine->target().profile_gemms(batch, reps, &b, launches);
        if (bytes) *bytes = b;
        return ms;
    } catch (const std::exception& e) {
        set_error(e.what());
        return -1.0;
    }
}

G4DENSE_API int g4dense_engine_set_gate(void* handle, double min_accept, int window) {
    clear_error();
    if (!handle) {
        set_error("Null handle");
        return -1;
    }
    auto* e = static_cast<EngineHandle*>(handle);
    e->gate_min_accept = min_accept;
    e->gate_window = window;
    return 0;
}

G4DENSE_API double g4dense_engine_time_pass(void* handle, int which, int batch, int pos, int reps) {
    clear_error();
    if (!handle || batch < 1 || batch > 128 || reps < 1 || pos < 0) {
        set_error("Invalid arguments");
        return -1.0;
    }
    try {
        auto* e = static_cast<EngineHandle*>(handle);
        if (which == 2) {  // one MTP drafter step (batch 1) with the target's KV up to pos
            g4b::DeviceModel* m = e->engine->mtp();
            if (!m) throw std::invalid_argument("no MTP drafter loaded");
            if (batch != 1 || pos < 1 || pos + 1 > e->engine->target().max_context())
                throw std::invalid_argument("an MTP step is one row at a position inside the target's KV");
            g4b::StepParams p{};
            p.base_pos = pos - 1;
            p.tokens[0] = 1;
            m->push_params(1, p, 1);
            m->enqueue(1, g4b::PassKind::MtpFirst, false, nullptr);  // warm (captures the graphs)
            m->enqueue(1, g4b::PassKind::MtpNext, false, nullptr);
            cudaEvent_t a, b;
            g4b::cuda_check(cudaEventCreate(&a), "event");
            g4b::cuda_check(cudaEventCreate(&b), "event");
            g4b::cuda_check(cudaEventRecord(a, m->stream()), "event");
            for (int r = 0; r < reps; ++r)
                m->enqueue(1, r == 0 ? g4b::PassKind::MtpFirst : g4b::PassKind::MtpNext, false, nullptr);
            g4b::cuda_check(cudaEventRecord(b, m->stream()), "event");
            g4b::cuda_check(cudaEventSynchronize(b), "event");
            float ms = 0.f;
            cudaEventElapsedTime(&ms, a, b);
            cudaEventDestroy(a);
            cudaEventDestroy(b);
            return (double)ms / reps;
        }
        g4b::DeviceModel* m = which == 0 ? &e->engine->target()
                                         : (e->engine->draft() ? &e->engine->draft()->model() : nullptr);
        if (!m) throw std::invalid_argument("no drafter loaded");
        if (which == 3) {  // chained one-row drafter steps from position pos, as a speculative round runs them
            if (batch != 1 || pos + 2 * reps + 2 > m->max_context())
                throw std::invalid_argument("drafter steps are one row, inside the KV capacity");
            g4b::StepParams p{};
            p.base_pos = pos;
            p.tokens[0] = 1;
            m->push_params(1, p, 1);
            for (int r = 0; r < 2; ++r) m->enqueue(1, g4b::PassKind::DraftStep, false, m->chain_dev());
            p.base_pos = pos;
            m->push_params(1, p, 1);
            cudaEvent_t a, b;
            g4b::cuda_check(cudaEventCreate(&a), "event");
            g4b::cuda_check(cudaEventCreate(&b), "event");
            g4b::cuda_check(cudaEventRecord(a, m->stream()), "event");
            for (int r = 0; r < reps; ++r) {
                if (r % 32 == 31) {  // the chain list holds 64 tokens: restart it between bursts
                    g4b::cuda_check(cudaEventRecord(b, m->stream()), "event");
                    g4b::cuda_check(cudaEventSynchronize(b), "event");
                    p.base_pos = pos + r;
                    m->push_params(1, p, 1);
                }
                m->enqueue(1, g4b::PassKind::DraftStep, false, m->chain_dev());
            }
            g4b::cuda_check(cudaEventRecord(b, m->stream()), "event");
            g4b::cuda_check(cudaEventSynchronize(b), "event");
            m->check_device_error();
            float ms = 0.f;
            cudaEventElapsedTime(&ms, a, b);
            cudaEventDestroy(a);
            cudaEventDestroy(b);
            return (double)ms / reps;
        }
        if (batch > m->max_rows()) throw std::invalid_argument("batch exceeds the model's rows per pass");
        if (pos + batch > m->max_context()) throw std::invalid_argument("pos + batch exceeds the KV capacity");
        std::vector<uint32_t> toks(batch, 1);
        m->run_plain(batch, pos, toks.data(), false);  // warm (captures the graph)
        cudaEvent_t a, b;
        g4b::cuda_check(cudaEventCreate(&a), "event");
        g4b::cuda_check(cudaEventCreate(&b), "event");
        g4b::cuda_check(cudaEventRecord(a, m->stream()), "event");
        for (int r = 0; r < reps; ++r) m->enqueue(batch, g4b::PassKind::Plain, false, nullptr);
        g4b::cuda_check(cudaEventRecord(b, m->stream()), "event");
        g4b::cuda_check(cudaEventSynchronize(b), "event");
        float ms = 0.f;
        cudaEventElapsedTime(&ms, a, b);
        cudaEventDestroy(a);
        cudaEventDestroy(b);
        return (double)ms / reps;
    } catch (const std::exception& ex) {
        set_error(ex.what());
        return -1.0;
    }
}

G4DENSE_API void g4dense_engine_stop(void* handle) {
    if (handle) static_cast<EngineHandle*>(handle)->cancel.store(true);
}

// ---- tokenizer ---------------------------------------------------------------------------

G4DENSE_API void* g4dense_tokenizer_open(const char* tokenizer_json_path, int arch) {
    clear_error();
    if (arch != 0 && arch != 1) {
        set_error("unknown tokenizer architecture (0 = Gemma-4, 1 = Muse-Glimmer)");
        return nullptr;
    }
    try {
        auto t = std::make_unique<TokHandle>();
        t->tok.load(tokenizer_json_path ? tokenizer_json_path : "");
        t->tok.set_arch(arch == 1 ? g4b::Tokenizer::Arch::MuseGlimmer : g4b::Tokenizer::Arch::Gemma4);
        return t.release();
    } catch (const std::exception& e) {
        set_error(e.what());
        return nullptr;
    }
}

G4DENSE_API void* g4dense_engine_tokenizer(void* handle) {
    return handle ? static_cast<EngineHandle*>(handle)->tok.get() : nullptr;
}

G4DENSE_API void g4dense_tokenizer_destroy(void* tok) {
    auto* t = static_cast<TokHandle*>(tok);
    if (t && !t->engine_owned) delete t;
}

G4DENSE_API int g4dense_tokenizer_encode(void* tok, const char* text, size_t len, int add_bos, unsigned int* out,
                                         int cap) {
    clear_error();
    if (!tok || (!text && len) || cap < 0 || (!out && cap)) {
        set_error("Invalid arguments");
        return -1;
    }
    try {
        const auto ids =
            static_cast<TokHandle*>(tok)->tok.encode(std::string_view(text ? text : "", len), add_bos != 0);
        if (ids.size() > (size_t)INT32_MAX) throw std::length_error("too many tokens");
        std::copy_n(ids.begin(), std::min(ids.size(), (size_t)cap), out);
        return (int)ids.size();
    } catch (const std::exception& e) {
        set_error(e.what());
        return -1;
    }
}

G4DENSE_API const char* g4dense_tokenizer_decode(void* tok, const unsigned int* ids, int n, int skip_special,
                                                 size_t* out_len) {
    clear_error();
    if (!tok || n < 0 || (!ids && n)) {
        set_error("Invalid arguments");
        return nullptr;
    }
    try {
        auto* t = static_cast<TokHandle*>(tok);
        return give(t->out, t->tok.decode(std::vector<uint32_t>(ids, ids + n), skip_special != 0), out_len);
    } catch (const std::exception& e) {
        set_error(e.what());
        return nullptr;
    }
}

G4DENSE_API const char* g4dense_tokenizer_decode_single(void* tok, unsigned int id, int skip_special,
                                                        size_t* out_len) {
    clear_error();
    if (!tok) {
        set_error("Invalid arguments");
        return nullptr;
    }
    auto* t = static_cast<TokHandle*>(tok);
    return guarded<const char*>(nullptr, [&] { return give(t->out, t->tok.decode_single(id, skip_special != 0), out_len); });
}

G4DENSE_API const char* g4dense_tokenizer_chat_template(void* tok, const char* messages_json) {
    clear_error();
    if (!tok || !messages_json) {
        set_error("Invalid arguments");
        return nullptr;
    }
    try {
        auto* t = static_cast<TokHandle*>(tok);
        return give(t->out, t->tok.chat_template(g4b::parse_chat_messages(messages_json)), nullptr);
    } catch (const std::exception& e) {
        set_error(e.what());
        return nullptr;
    }
}

G4DENSE_API int g4dense_tokenizer_special_ids(void* tok, unsigned int* out6) {
    if (!tok || !out6) return -1;
    const g4b::Tokenizer& t = static_cast<TokHandle*>(tok)->tok;
    const unsigned int v[6] = {t.bos(), t.eos(), t.pad(), t.unk(), t.end_of_turn(), t.vocab_size()};
    std::memcpy(out6, v, sizeof(v));
    return 0;
}

G4DENSE_API int g4dense_tokenizer_stop_ids(void* tok, unsigned int* out, int cap) {
    if (!tok || cap < 0 || (!out && cap)) return 0;
    const auto& s = static_cast<TokHandle*>(tok)->tok.stop_ids();
    std::copy_n(s.begin(), std::min(s.size(), (size_t)cap), out);
    return (int)s.size();
}

G4DENSE_API int g4dense_tokenizer_byte_value(void* tok, unsigned int id, unsigned char* value) {
    uint8_t b = 0;
    if (!tok || !static_cast<TokHandle*>(tok)->tok.byte_value(id, b)) return 0;
    if (value) *value = b;
    return 1;
}

G4DENSE_API int g4dense_tokenizer_is_special(void* tok, unsigned int id) {
    return tok && static_cast<TokHandle*>(tok)->tok.is_special(id) ? 1 : 0;
}

G4DENSE_API void* g4dense_detokenizer_create(void* tok, int skip_special) {
    clear_error();
    if (!tok) {
        set_error("null tokenizer");
        return nullptr;
    }
    return guarded<void*>(nullptr, [&] { return new DetokHandle(static_cast<TokHandle*>(tok)->tok, skip_special != 0); });
}

G4DENSE_API const char* g4dense_detokenizer_push(void* detok, unsigned int id, size_t* out_len) {
    if (!detok) return nullptr;
    auto* d = static_cast<DetokHandle*>(detok);
    return guarded<const char*>(nullptr, [&] { return give(d->out, d->d.push(id), out_len); });
}

G4DENSE_API const char* g4dense_detokenizer_finish(void* detok, size_t* out_len) {
    if (!detok) return nullptr;
    auto* d = static_cast<DetokHandle*>(detok);
    return guarded<const char*>(nullptr, [&] { return give(d->out, d->d.finish(), out_len); });
}

G4DENSE_API void g4dense_detokenizer_destroy(void* detok) { delete static_cast<DetokHandle*>(detok); }

G4DENSE_API void* g4dense_stop_matcher_create(const char* const* stops, int n) {
    clear_error();
    if (n < 0 || (!stops && n)) {
        set_error("Invalid arguments");
        return nullptr;
    }
    return guarded<void*>(nullptr, [&] {
        std::vector<std::string> v;
        for (int i = 0; i < n; ++i) v.emplace_back(stops[i] ? stops[i] : "");
        auto m = std::make_unique<StopHandle>();
        m->m = g4b::StreamingStopMatcher(std::move(v));
        return static_cast<void*>(m.release());
    });
}

G4DENSE_API const char* g4dense_stop_matcher_push(void* m, const char* text, size_t len, size_t* out_len) {
    if (!m || (!text && len)) return nullptr;
    auto* h = static_cast<StopHandle*>(m);
    return guarded<const char*>(nullptr,
                                [&] { return give(h->out, h->m.push(std::string_view(text ? text : "", len)), out_len); });
}

G4DENSE_API const char* g4dense_stop_matcher_finish(void* m, size_t* out_len) {
    if (!m) return nullptr;
    auto* h = static_cast<StopHandle*>(m);
    return guarded<const char*>(nullptr, [&] { return give(h->out, h->m.finish(), out_len); });
}

G4DENSE_API int g4dense_stop_matcher_stopped(void* m, const char** matched) {
    if (!m) return 0;
    auto* h = static_cast<StopHandle*>(m);
    if (matched) *matched = h->m.matched().c_str();
    return h->m.stopped() ? 1 : 0;
}

G4DENSE_API void g4dense_stop_matcher_destroy(void* m) { delete static_cast<StopHandle*>(m); }

G4DENSE_API const char* g4dense_utf8_repair(const char* in, size_t len, int flush_all, size_t* consumed,
                                            size_t* out_len) {
    thread_local std::string buf;
    return guarded<const char*>(nullptr, [&] {
        std::string out;
        const size_t used = g4b::utf8_repair(std::string_view(in ? in : "", in ? len : 0), flush_all != 0, out);
        if (consumed) *consumed = used;
        return give(buf, std::move(out), out_len);
    });
}

G4DENSE_API int g4dense_container_validate(const char* path) {
    clear_error();
    try {
        if (!path) throw std::invalid_argument("container path is NULL");
        std::ifstream f(path, std::ios::binary | std::ios::ate);
        if (!f) throw g4b::G4DenseFormatError(std::string("cannot open container ") + path);
        const uint64_t size = static_cast<uint64_t>(f.tellg());
        unsigned char raw[4096];
        static_assert(sizeof(raw) == sizeof(g4b::G4DenseHeader) && sizeof(raw) == sizeof(g4b::G4MtpHeader),
                      "both headers fill one 4096-byte page");
        if (size < sizeof(raw)) throw g4b::G4DenseFormatError("container file too small for header");
        f.seekg(0);
        if (!f.read(reinterpret_cast<char*>(raw), sizeof(raw)))
            throw g4b::G4DenseFormatError(std::string("cannot read the header of ") + path);
        uint32_t magic;
        std::memcpy(&magic, raw, sizeof magic);
        if (magic == g4b::G4MtpHeader::kMagic) {
            g4b::G4MtpHeader h;
            std::memcpy(&h, raw, sizeof h);
            g4b::validate_mtp_header(h, size);
            return 2;
        }
        g4b::G4DenseHeader h;
        std::memcpy(&h, raw, sizeof h);
        g4b::validate_header(h, size);
        return 1;
    } catch (const std::exception& e) {
        set_error(e.what());
        return -1;
    }
}

}  // extern "C"
