// The public C++ interfaces (include/g4dense/*.hpp): the reference's ForwardRunner, DraftRuntime,
// SpeculativeCoordinator and sampling functions, backed by the engine's DeviceModel / Engine.
#include <cuda_runtime.h>

#include <chrono>
#include <cstdio>
#include <cstring>
#include <stdexcept>

#include "g4dense/device_context.hpp"
#include "g4dense/draft_runtime.hpp"
#include "g4dense/runner.hpp"
#include "g4dense/sampling.hpp"
#include "g4dense/speculator.hpp"
#include "runner.h"
#include "sampling.h"
#include "tokenizer_impl.h"
#ifdef G4B_HAVE_NCCL
#include <nccl.h>
#endif

namespace g4dense {

namespace {
g4b::SamplingParams to_internal(const SamplingParams& p) {
    g4b::SamplingParams q;
    q.temperature = p.temperature;
    q.top_p = p.top_p;
    q.top_k = p.top_k;
    q.repetition_penalty = p.repetition_penalty;
    q.has_seed = p.has_seed;
    q.seed = p.seed;
    return q;
}

void use_device(int dev) {
    if (dev >= 0) g4b::cuda_check(cudaSetDevice(dev), "cudaSetDevice");
}

uint32_t file_magic(const std::string& path) {
    uint32_t magic = 0;
    if (FILE* f = std::fopen(path.c_str(), "rb")) {
        if (std::fread(&magic, 4, 1, f) != 1) magic = 0;
        std::fclose(f);
    }
    return magic;
}
}  // namespace

// ------------------------------------------------------------------------------- DeviceContext

struct DeviceContext::Impl {
    int device = 0, rank = 0, size = 1;
    void* comm = nullptr;
};

DeviceContext::DeviceContext() : impl_(new Impl) {}

DeviceContext::~DeviceContext() {
#ifdef G4B_HAVE_NCCL
    if (impl_->comm) ncclCommDestroy((ncclComm_t)impl_->comm);
#endif
}

std::shared_ptr<DeviceContext> DeviceContext::create(int device, int tp_rank, int tp_size, const void* nccl_id) {
    if (tp_size < 1 || tp_rank < 0 || tp_rank >= tp_size) throw std::invalid_argument("DeviceContext: bad rank/size");
    std::shared_ptr<DeviceContext> c(new DeviceContext());
    if (device < 0) g4b::cuda_check(cudaGetDevice(&device), "cudaGetDevice");
    use_device(device);
    g4b::cuda_check(cudaFree(nullptr), "device context");  // creates the primary context now
    c->impl_->device = device;
    c->impl_->rank = tp_rank;
    c->impl_->size = tp_size;
    if (tp_size > 1) {
#ifdef G4B_HAVE_NCCL
        if (!nccl_id) throw std::invalid_argument("DeviceContext: tensor parallelism needs an NCCL unique id");
        ncclUniqueId id;
        std::memcpy(&id, nccl_id, sizeof(id));
        ncclComm_t comm;
        if (ncclCommInitRank(&comm, tp_size, id, tp_rank) != ncclSuccess)
            throw std::runtime_error("DeviceContext: ncclCommInitRank failed");
        c->impl_->comm = comm;
#else
        throw std::runtime_error("DeviceContext: built without NCCL");
#endif
    }
    return c;
}

void DeviceContext::nccl_unique_id(void* out128) {
#ifdef G4B_HAVE_NCCL
    ncclUniqueId id;
    if (ncclGetUniqueId(&id) != ncclSuccess) throw std::runtime_error("ncclGetUniqueId failed");
    std::memcpy(out128, &id, sizeof(id));
#else
    (void)out128;
    throw std::runtime_error("built without NCCL");
#endif
}

int DeviceContext::device() const { return impl_->device; }
int DeviceContext::tp_rank() const { return impl_->rank; }
int DeviceContext::tp_size() const { return impl_->size; }
void* DeviceContext::nccl_comm() const { return impl_->comm; }

// ------------------------------------------------------------------------------- sampling

void validate_sampling(const SamplingParams& p) { g4b::validate_sampling(to_internal(p)); }
uint64_t splitmix64(uint64_t x) { return g4b::splitmix64(x); }
uint64_t seed_for(const SamplingParams& p, int position) { return g4b::seed_for(to_internal(p), position); }
void apply_repetition_penalty(float* logits, uint32_t vocab, const std::vector<uint32_t>& history, float penalty,
                              float softcap) {
    g4b::apply_repetition_penalty(logits, vocab, history, penalty, softcap);
}
uint32_t sample_token(const float* logits, uint32_t vocab, const SamplingParams& p, uint64_t seed) {
    return g4b::sample_token(logits, vocab, to_internal(p), seed);
}

// ------------------------------------------------------------------------------- speculator

struct SpeculativeCoordinator::Impl {
    g4b::SpeculativeCoordinator sc;
};

SpeculativeCoordinator::SpeculativeCoordinator() : impl_(new Impl) {}
SpeculativeCoordinator::~SpeculativeCoordinator() = default;

SpeculativeEvaluation SpeculativeCoordinator::evaluate_verification(
    const std::vector<uint32_t>& draft_tokens, const std::vector<const float*>& target_logits_per_pos,
    uint32_t vocab_size, const SamplingParams& sampling, uint64_t base_seed,
    const std::vector<std::vector<float>>& draft_logits) {
    const g4b::SpeculativeEvaluation e = impl_->sc.evaluate_verification(
        draft_tokens, target_logits_per_pos, vocab_size, to_internal(sampling), base_seed, draft_logits);
    SpeculativeEvaluation r;
    r.accepted_tokens = e.accepted_tokens;
    r.num_accepted = e.num_accepted;
    r.total_drafted = e.total_drafted;
    r.bonus_token_sampled = e.bonus_token_sampled;
    r.bonus_token = e.bonus_token;
    r.acceptance_rate = e.acceptance_rate;
    return r;
}
uint64_t SpeculativeCoordinator::total_draft_tokens() const { return impl_->sc.total_draft_tokens(); }
uint64_t SpeculativeCoordinator::total_accepted_tokens() const { return impl_->sc.total_accepted_tokens(); }

// ------------------------------------------------------------------------------- DraftRuntime

struct DraftRuntime::Impl {
    std::shared_ptr<DeviceContext> ctx;
    std::unique_ptr<g4b::DeviceModel> model;
    size_t consumed = 0;   // context tokens already in the drafter's KV cache
    size_t forwarded = 0;  // positions the drafter has forwarded (its cache's true extent)
};

DraftRuntime::DraftRuntime() : impl_(new Impl) {}
DraftRuntime::~DraftRuntime() = default;

bool DraftRuntime::load_model(const std::string& path, std::shared_ptr<DeviceContext> ctx, int max_context) {
    if (!ctx) throw std::invalid_argument("DraftRuntime: a DeviceContext is required");
    if (FILE* f = std::fopen(path.c_str(), "rb")) {
        std::fclose(f);
    } else {
        impl_->model.reset();
        throw std::runtime_error("DraftRuntime: draft model container not found: " + path);
    }
    use_device(ctx->device());
    g4b::ModelOptions o;
    o.max_context = max_context;
    auto m = std::make_unique<g4b::DeviceModel>(o);
    m->load_container(path);
    impl_->model = std::move(m);
    impl_->ctx = std::move(ctx);
    impl_->consumed = impl_->forwarded = 0;
    return true;
}

bool DraftRuntime::is_loaded() const { return impl_->model != nullptr; }

void DraftRuntime::reset() {
    if (impl_->model) impl_->model->clear_kv();
    impl_->consumed = impl_->forwarded = 0;
}

void DraftRuntime::accept(size_t accepted_context_length) {
    impl_->consumed = std::min(accepted_context_length, impl_->forwarded);
}

DraftResult DraftRuntime::generate_draft_tokens(const std::vector<uint32_t>& context, uint32_t k,
                                                const SamplingParams& sampling) {
    const auto t0 = std::chrono::steady_clock::now();
    DraftResult res;
    if (!impl_->model || k == 0 || context.empty()) return res;
    use_device(impl_->ctx->device());
    g4b::DeviceModel& m = *impl_->model;
    const uint32_t V = m.header().vocab_size;
    const g4b::SamplingParams sp = to_internal(sampling);
    if (impl_->consumed > context.size()) {
        m.clear_kv();
        impl_->consumed = 0;
    }
    // Unseen context before the last token, in passes of up to 16 positions (batched rows
    // compute what single positions do).
    while (impl_->consumed + 1 < context.size()) {
        const int rows = (int)std::min<size_t>(context.size() - 1 - impl_->consumed, g4b::kBatchRows);
        m.run_plain(rows, (int)impl_->consumed, context.data() + impl_->consumed, false);
        impl_->consumed += rows;
    }
    std::vector<float> logits(V);
    uint32_t cur = context.back();
    int pos = (int)impl_->consumed;
    for (uint32_t step = 0; step < k; ++step) {
        m.run_plain(1, pos++, &cur, true);
        m.logits_to_host(0, 1, logits.data());
        const uint64_t seed = g4b::splitmix64(sp.has_seed ? (sp.seed + step) : (1337 + step));
        const uint32_t cand = g4b::sample_token(logits.data(), V, sp, seed);
        res.draft_tokens.push_back(cand);
        res.draft_logits.push_back(logits);
        cur = cand;
    }
    impl_->forwarded = (size_t)pos;
    impl_->consumed = context.size();
    res.draft_time_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    return res;
}

// ------------------------------------------------------------------------------- ForwardRunner

struct ForwardRunner::Impl {
    std::shared_ptr<DeviceContext> ctx;
    std::string path;
    uint32_t max_context = 4096;
    std::unique_ptr<g4b::Engine> engine;
    std::shared_ptr<Tokenizer> tok;
    void require() const {
        if (!engine) throw std::runtime_error("ForwardRunner: call initialize() first");
    }
    // The runner decides the tokenizer's architecture from the container (src/runner.cpp:265).
    void sync_arch() {
        if (tok && engine)
            tok->set_architecture(engine->target().header().arch_type == 1 ? ModelArch::MUSE_GLIMMER
                                                                           : ModelArch::GEMMA4);
    }
};

ForwardRunner::ForwardRunner(std::shared_ptr<DeviceContext> ctx, const std::string& container_path)
    : impl_(new Impl) {
    if (!ctx) throw std::invalid_argument("ForwardRunner: a DeviceContext is required");
    impl_->ctx = std::move(ctx);
    impl_->path = container_path;
}

ForwardRunner::ForwardRunner(std::shared_ptr<DeviceContext> ctx, std::shared_ptr<Tokenizer> tokenizer,
                             const std::string& container_path)
    : ForwardRunner(std::move(ctx), container_path) {
    impl_->tok = std::move(tokenizer);
}

void ForwardRunner::set_tokenizer(std::shared_ptr<Tokenizer> tokenizer) {
    impl_->tok = std::move(tokenizer);
    impl_->sync_arch();
}

ForwardRunner::~ForwardRunner() {
    if (impl_->engine) use_device(impl_->ctx->device());
    impl_->engine.reset();
}

void ForwardRunner::set_max_context(uint32_t n) { impl_->max_context = n; }
uint32_t ForwardRunner::max_context() const {
    return impl_->engine ? (uint32_t)impl_->engine->target().max_context() : 0u;
}

void ForwardRunner::initialize() {
    use_device(impl_->ctx->device());
    g4b::ModelOptions o;
    o.max_context = (int)impl_->max_context;
    o.rank = impl_->ctx->tp_rank();
    o.tp = impl_->ctx->tp_size();
    o.nccl_comm = impl_->ctx->nccl_comm();
    auto t = std::make_unique<g4b::DeviceModel>(o);
    t->load_container(impl_->path);
    impl_->engine = std::make_unique<g4b::Engine>(std::move(t));
    impl_->sync_arch();
}

void ForwardRunner::forward_batch(const uint32_t* ids, uint32_t batch, uint32_t base, float* out_logits,
                                  bool all_positions) {
    impl_->require();
    use_device(impl_->ctx->device());
    impl_->engine->forward_batch(ids, batch, base, out_logits, all_positions);
}

void ForwardRunner::forward_single_token(uint32_t token_id, uint32_t position, float* out_logits) {
    forward_batch(&token_id, 1, position, out_logits, false);
}

void ForwardRunner::generate(const std::string& prompt, const GenerationOptions& o, TokenCallback on_token,
                             std::atomic<bool>* cancel) {
    if (!impl_->tok || !impl_->tok->is_loaded())
        throw std::runtime_error("ForwardRunner::generate: Tokenizer is not loaded or missing");
    impl_->require();
    use_device(impl_->ctx->device());
    const g4b::Tokenizer& tk = impl_->tok->impl_->t;
    // The template emits the literal "<bos>", so the templated text is encoded without another.
    const std::vector<uint32_t> ids =
        o.use_chat_template ? tk.encode(tk.chat_template({{"user", prompt}}), false) : tk.encode(prompt, true);
    if (ids.empty()) throw std::runtime_error("ForwardRunner::generate: prompt encoded to empty token sequence");
    g4b::Engine& e = *impl_->engine;
    g4b::GenerationOptions g;
    g.max_tokens = o.max_tokens;
    g.sampling = to_internal(o.sampling);
    g.speculative_enabled = o.speculative_enabled && (e.draft() || e.mtp());
    g.draft_k = o.draft_k;
    g.stop_token = o.stop_token;
    g.stop_tokens = tk.stop_ids();
    g4b::TokenCallback cb;
    if (on_token) cb = [&](uint32_t t) { return on_token(t, tk.decode_single(t)); };
    e.generate(ids, g, cb, cancel);
}

std::vector<uint32_t> ForwardRunner::generate_tokens(const std::vector<uint32_t>& prompt, const GenerationOptions& o,
                                                     TokenCallback on_token, std::atomic<bool>* cancel) {
    impl_->require();
    use_device(impl_->ctx->device());
    g4b::Engine& e = *impl_->engine;
    g4b::GenerationOptions g;
    g.max_tokens = o.max_tokens;
    g.sampling = to_internal(o.sampling);
    g.speculative_enabled = o.speculative_enabled && (e.draft() || e.mtp());
    g.draft_k = o.draft_k;
    g.stop_token = o.stop_token;
    g4b::TokenCallback cb;
    const Tokenizer* tok = impl_->tok && impl_->tok->is_loaded() ? impl_->tok.get() : nullptr;
    if (on_token)
        cb = [&on_token, tok](uint32_t t) { return on_token(t, tok ? tok->decode_single(t) : std::string()); };
    return e.generate(prompt, g, cb, cancel);
}

std::vector<RoundRecord> ForwardRunner::last_rounds() const {
    std::vector<RoundRecord> out;
    if (!impl_->engine) return out;
    const std::vector<int>& ri = impl_->engine->last_stats().round_info;
    for (size_t i = 0; i + 2 < ri.size(); i += 3) out.push_back({ri[i], ri[i + 1], ri[i + 2]});
    return out;
}

void ForwardRunner::switch_memory_tier(uint32_t) {}

void ForwardRunner::reset_kv_cache() {
    impl_->require();
    use_device(impl_->ctx->device());
    impl_->engine->target().clear_kv();
    g4b::cuda_check(cudaStreamSynchronize(impl_->engine->target().stream()), "reset_kv_cache");
}

bool ForwardRunner::load_draft_model(const std::string& path) {
    impl_->require();
    use_device(impl_->ctx->device());
    g4b::DeviceModel& T = impl_->engine->target();
    g4b::ModelOptions o;
    o.max_context = T.max_context();
    o.kv_bf16 = T.options().kv_bf16;
    if (file_magic(path) == g4b::G4MtpHeader::kMagic) {
        // The MTP assistant reads the target's KV rings and hidden states, on its stream.
        if (T.options().tp != 1) throw std::invalid_argument("the MTP drafter runs without tensor parallelism");
        T.enable_hidden_out();
        o.prefill_tc = false;
        o.stream = T.stream();
        auto d = std::make_unique<g4b::DeviceModel>(o);
        d->load_mtp(path, T);
        impl_->engine->set_mtp(std::move(d));
    } else {
        auto d = std::make_unique<g4b::DeviceModel>(o);
        d->load_container(path);
        impl_->engine->set_draft(std::move(d));
    }
    return true;
}

bool ForwardRunner::has_draft_model() const {
    return impl_->engine && (impl_->engine->draft() != nullptr || impl_->engine->mtp() != nullptr);
}

uint32_t ForwardRunner::vocab_size() const {
    impl_->require();
    return impl_->engine->target().header().vocab_size;
}
uint32_t ForwardRunner::num_layers() const {
    impl_->require();
    return impl_->engine->target().header().num_layers;
}
uint32_t ForwardRunner::d_model() const {
    impl_->require();
    return impl_->engine->target().header().d_model;
}

std::string ForwardRunner::device_name() const {
    cudaDeviceProp p{};
    if (cudaGetDeviceProperties(&p, impl_->ctx->device()) != cudaSuccess) return std::string();
    return p.name;
}

}  // namespace g4dense
