// The target model's forward pass and generation loop, the reference's ForwardRunner
// (include/g4dense/runner.hpp:25-157, src/runner.cpp:906-2347), with the model fully resident on
// one B200 (or tensor-parallel over the ranks of the DeviceContext). The reference's Vulkan,
// streaming and tier machinery has no counterpart: everything is resident, so tiers and the layer
// cache are gone. Text goes through the Tokenizer given at construction (or set_tokenizer);
// generate_tokens takes token ids directly.
#pragma once
#include <atomic>
#include <cstdint>
#include <functional>
#include <memory>
#include <string>
#include <vector>

#include "g4dense/device_context.hpp"
#include "g4dense/sampling.hpp"
#include "g4dense/tokenizer.hpp"

namespace g4dense {

struct GenerationOptions {
    int max_tokens{512};
    SamplingParams sampling{};
    bool speculative_enabled{false};  // off by default, as in the reference
    uint32_t draft_k{6};              // verify width K (K - 1 drafts); the B200 path takes 2..16
    uint32_t active_tier_id{1};       // accepted and ignored: every layer is resident
    bool use_chat_template{true};     // generate(): wrap the prompt in one user turn (generate_tokens: unused)
    int64_t stop_token{-1};           // additive: < 0 = none
};

// Called once per emitted token; returning false stops generation. `piece` is
// Tokenizer::decode_single(token) ("" from generate_tokens when the runner has no tokenizer).
using TokenCallback = std::function<bool(uint32_t token, const std::string& piece)>;

// Per-round record of speculative decoding: (drafted, accepted, emitted).
struct RoundRecord {
    int drafted, accepted, emitted;
};

class G4DENSE_CXX_API ForwardRunner {
   public:
    ForwardRunner(std::shared_ptr<DeviceContext> ctx, const std::string& container_path);
    // The reference's constructor (include/g4dense/runner.hpp:60-62): the tokenizer serves generate().
    ForwardRunner(std::shared_ptr<DeviceContext> ctx, std::shared_ptr<Tokenizer> tokenizer,
                  const std::string& container_path);
    ~ForwardRunner();
    ForwardRunner(const ForwardRunner&) = delete;
    ForwardRunner& operator=(const ForwardRunner&) = delete;

    // Loads the container onto the device (validating it) and sizes the KV cache. Throws on a
    // missing or malformed file.
    void initialize();
    // KV capacity of full-attention layers; call before initialize() (the reference's rule).
    void set_max_context(uint32_t n);
    uint32_t max_context() const;

    // One pass over `batch` consecutive positions from base_position (1..128; above 16 only the
    // last row's logits exist). out_logits (host, may be null) receives the last position's
    // logits, or all batch rows' when all_positions.
    void forward_batch(const uint32_t* token_ids, uint32_t batch, uint32_t base_position, float* out_logits,
                       bool all_positions = false);
    void forward_single_token(uint32_t token_id, uint32_t position, float* out_logits);

    // The reference's text entry point (src/runner.cpp:2060-2347): the prompt is wrapped in one
    // user turn of the chat template and encoded without another <bos> (use_chat_template), or
    // encoded with <bos>; generation stops after any of the tokenizer's stop ids, and on_token
    // receives each emitted token with its decode_single piece. Throws std::runtime_error without
    // a loaded tokenizer.
    void generate(const std::string& prompt, const GenerationOptions& options, TokenCallback on_token,
                  std::atomic<bool>* cancel_flag = nullptr);
    // Sets the tokenizer (its architecture follows the container once initialized).
    void set_tokenizer(std::shared_ptr<Tokenizer> tokenizer);
    // Generation from token ids: prompt prefill, then the speculative round loop (when enabled and
    // a drafter is loaded) or the plain loop. Stops only on options.stop_token (no tokenizer stop
    // ids). Returns the emitted tokens.
    std::vector<uint32_t> generate_tokens(const std::vector<uint32_t>& prompt_ids, const GenerationOptions& options,
                                          TokenCallback on_token = nullptr, std::atomic<bool>* cancel_flag = nullptr);
    // Round records of the last generate_tokens call.
    std::vector<RoundRecord> last_rounds() const;

    // Accepted for interface parity: every layer is resident, so there is nothing to switch.
    void switch_memory_tier(uint32_t tier_id);
    // Forgets every cached key/value so an independent sequence can run from position 0
    // (generate_tokens does this itself).
    void reset_kv_cache();
    // Loads a drafter (.g4dense, or an MTP assistant .g4mtp recognised by its magic) on this
    // runner's device. Returns true on success; throws on a malformed file.
    bool load_draft_model(const std::string& path);
    bool has_draft_model() const;

    uint32_t vocab_size() const;
    uint32_t num_layers() const;
    uint32_t d_model() const;
    std::string device_name() const;

   private:
    struct Impl;
    std::unique_ptr<Impl> impl_;
};

}  // namespace g4dense
