// The decode engine: ForwardRunner::forward_batch / generate (include/g4dense/runner.hpp:
// 100-157, src/runner.cpp:2061-2347), DraftRuntime (include/g4dense/draft_runtime.hpp:19-54)
// and the speculative round loop, over B200 DeviceModels. Prompts are token ids (the
// reference's tokenizer and chat template sit outside this path).
#pragma once
#include <atomic>
#include <cstdint>
#include <functional>
#include <memory>
#include <string>
#include <vector>

#include "model.h"
#include "sampling.h"

namespace g4b {

// Widest verify batch: the reference caps K at kGemmMaxBatch = 8
// (include/g4dense/vk_pipeline.hpp:21); the B200 kernels take 16 rows, which BASELINE's
// k = 8 configuration (K = 9) needs.
constexpr uint32_t kMaxDraftWidth = 16;

struct GenerationOptions {
    int max_tokens{512};
    SamplingParams sampling{};
    bool speculative_enabled{false};  // off by default, as in the reference
    uint32_t draft_k{6};              // verify width K (K-1 drafts), clamped to [2, 8]
    int64_t stop_token{-1};           // < 0: no stop token
    std::vector<uint32_t> stop_tokens;  // the tokenizer's stop ids (text generation)
    double gate_min_accept{0.45};     // adaptive gate (src/runner.cpp:2188-2195)
    int gate_window{24};
    // Config-3 "oracle drafter": the drafter model still runs its steps (cost), but the
    // proposals replay `replay` (the target's own greedy stream after the prompt) with
    // i.i.d. injected mismatches at `mismatch_rate`.
    std::vector<uint32_t> replay;
    double mismatch_rate{0.0};
    uint64_t mismatch_seed{0};
    // Non-speculative sampled decoding draws each token on the device (sample.cu) instead of
    // copying the logits row to the host; a repetition penalty keeps the host path.
    bool device_sampling{true};
};

struct GenStats {
    uint64_t drafted{0}, accepted{0}, rounds{0}, gated_steps{0}, emitted{0};
    double ttft_ms{0}, total_ms{0}, decode_ms{0}, draft_ms{0}, verify_ms{0};
    double decode_gpu_ms{0};        // device time from the end of prefill to the last token (CUDA events)
    uint64_t launches{0};           // kernels enqueued by this generation (target + drafter)
    uint64_t h2d_bytes{0}, d2h_bytes{0};  // host<->device copies of this generation
    bool gated{false};
    uint32_t draft_k{0};          // verify width of the speculative rounds (0 without speculation)
    uint64_t context_tokens{0};   // prompt + emitted tokens held by the KV cache at the end
    std::vector<int> round_info;  // (drafted, accepted, emitted) per verify round
    int stop_reason{0};           // 0 max_tokens, 1 stop token, 2 callback, 3 cancelled
};

using TokenCallback = std::function<bool(uint32_t token)>;

// DraftRuntime: a second DeviceModel on the target's stream plus the bookkeeping of how much
// of the context its KV cache holds (src/draft_runtime.cpp:46-103).
class DraftRuntime {
   public:
    explicit DraftRuntime(std::unique_ptr<DeviceModel> m) : model_(std::move(m)) {}
    DeviceModel& model() { return *model_; }
    void reset() { consumed_ = 0; }
    size_t consumed() const { return consumed_; }
    // Feeds context[consumed, n-1) so the cache holds every token before the pending one.
    void catch_up(const std::vector<uint32_t>& context);
    // accept(): the reference sets consumed to the kept length; it is capped here at what the
    // drafter actually forwarded, so a fully accepted round feeds its last draft next round.
    void accept(size_t accepted_context_length, size_t forwarded) {
        consumed_ = std::min(accepted_context_length, forwarded);
    }
    void set_consumed(size_t c) { consumed_ = c; }

   private:
    std::unique_ptr<DeviceModel> model_;
    size_t consumed_{0};
};

class Engine {
   public:
    explicit Engine(std::unique_ptr<DeviceModel> target) : target_(std::move(target)) {}
    ~Engine() {
        for (auto e : order_ev_)
            if (e) cudaEventDestroy(e);
    }
    Engine(const Engine&) = delete;
    Engine& operator=(const Engine&) = delete;
    DeviceModel& target() { return *target_; }
    DraftRuntime* draft() { return draft_.get(); }
    void set_draft(std::unique_ptr<DeviceModel> d) { draft_ = std::make_unique<DraftRuntime>(std::move(d)); }
    // The MTP assistant drafter: a DeviceModel loaded with load_mtp*, on the target's stream.
    void set_mtp(std::unique_ptr<DeviceModel> m) { mtp_ = std::move(m); }
    DeviceModel* mtp() { return mtp_.get(); }
    // Tensor parallelism: the drafter lives on rank 0 only. The other ranks set this and take
    // each round's drafts (and, when sampling, its acceptance result) by broadcast from rank 0.
    void set_remote_draft(bool on) { remote_draft_ = on; }
    bool has_drafter() const { return draft_ || mtp_ || remote_draft_; }

    // One pass over `batch` consecutive positions from base_position (runner.hpp:110-111).
    // out_logits (host) receives the last row's logits, or all rows' when all_positions.
    void forward_batch(const uint32_t* token_ids, uint32_t batch, uint32_t base_position, float* out_logits,
                       bool all_positions = false);
    // Generation from token ids; returns the emitted tokens.
    std::vector<uint32_t> generate(const std::vector<uint32_t>& prompt, const GenerationOptions& opt,
                                   const TokenCallback& on_token, const std::atomic<bool>* cancel = nullptr);
    const GenStats& last_stats() const { return stats_; }
    std::string telemetry_json() const;

   private:
    // Runs the prompt; returns the greedy next token. last_logits (may be null) receives the
    // last position's logits on sampled runs; last_row_ names their row on the device.
    uint32_t prefill(const std::vector<uint32_t>& tokens, const GenerationOptions& opt, std::vector<float>* last_logits);
    // Makes `to` wait for the work queued on `from` so far.
    void order(cudaStream_t from, cudaStream_t to);

    std::unique_ptr<DeviceModel> target_;
    std::unique_ptr<DraftRuntime> draft_;
    std::unique_ptr<DeviceModel> mtp_;
    bool remote_draft_ = false;
    int mtp_row_ = 0;  // row of the target's normed hidden states the next MTP round starts from
    cudaEvent_t order_ev_[2] = {nullptr, nullptr};
    int order_i_ = 0;
    int last_row_ = 0;  // device logits row of the last pass's final position
    SpeculativeCoordinator speculator_;
    GenStats stats_;
};

}  // namespace g4b
