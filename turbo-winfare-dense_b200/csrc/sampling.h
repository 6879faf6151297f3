// Host-side sampling and speculative acceptance with the reference's semantics:
// SamplingParams / validate_sampling / splitmix64 / seed_for / sample_token
// (include/g4dense/sampling.hpp:9-27, src/sampling.cpp:232-369) and
// SpeculativeCoordinator::evaluate_verification (src/speculator.cpp:34-153). Greedy decoding
// runs on the device (head.cu); these serve the sampled path, whose random draws must match
// the reference's host RNG streams bit for bit.
#pragma once
#include <cstdint>
#include <vector>

namespace g4b {

struct SamplingParams {
    float temperature{0.0f};
    float top_p{1.0f};
    int top_k{0};
    float repetition_penalty{1.0f};
    bool has_seed{false};
    uint64_t seed{0};
    bool is_greedy() const { return temperature <= 0.0f && repetition_penalty == 1.0f; }
};

void validate_sampling(const SamplingParams& p);  // throws std::invalid_argument
uint64_t splitmix64(uint64_t x);
uint64_t seed_for(const SamplingParams& p, int position);
void apply_repetition_penalty(float* logits, uint32_t vocab, const std::vector<uint32_t>& history, float penalty,
                              float softcap);
uint32_t sample_token(const float* logits, uint32_t vocab, const SamplingParams& p, uint64_t seed);

struct SpeculativeEvaluation {
    std::vector<uint32_t> accepted_tokens;  // accepted drafts + the correction/bonus token
    uint32_t num_accepted{0};
    uint32_t total_drafted{0};
    bool bonus_token_sampled{false};
    uint32_t bonus_token{0};
    double acceptance_rate{0.0};
};

class SpeculativeCoordinator {
   public:
    SpeculativeEvaluation evaluate_verification(const std::vector<uint32_t>& draft_tokens,
                                                const std::vector<const float*>& target_logits_per_pos,
                                                uint32_t vocab_size, const SamplingParams& sampling,
                                                uint64_t base_seed,
                                                const std::vector<std::vector<float>>& draft_logits = {});
    uint64_t total_draft_tokens() const { return total_draft_; }
    uint64_t total_accepted_tokens() const { return total_accepted_; }

   private:
    uint64_t total_draft_{0}, total_accepted_{0};
};

}  // namespace g4b
