// Speculative acceptance, the reference's SpeculativeCoordinator (include/g4dense/speculator.hpp:
// 10-31, src/speculator.cpp:34-153): greedy acceptance while each draft equals the target's argmax
// at its position, then the target's token (correction or bonus); sampled acceptance by the ratio
// test p/q with an mt19937_64 draw seeded from base_seed and a residual draw on rejection.
#pragma once
#include <cstdint>
#include <memory>
#include <vector>

#include "g4dense/sampling.hpp"

namespace g4dense {

struct SpeculativeEvaluation {
    std::vector<uint32_t> accepted_tokens;  // accepted drafts + the correction or bonus token
    uint32_t num_accepted{0};
    uint32_t total_drafted{0};
    bool bonus_token_sampled{false};
    uint32_t bonus_token{0};
    double acceptance_rate{0.0};
};

class G4DENSE_CXX_API SpeculativeCoordinator {
   public:
    SpeculativeCoordinator();
    ~SpeculativeCoordinator();
    // target_logits_per_pos: draft_tokens.size() + 1 rows of vocab_size fp32 logits (the verify
    // pass over the pending token and the drafts); draft_logits: the drafter's logits per draft
    // (sampled acceptance only).
    SpeculativeEvaluation evaluate_verification(const std::vector<uint32_t>& draft_tokens,
                                                const std::vector<const float*>& target_logits_per_pos,
                                                uint32_t vocab_size, const SamplingParams& sampling,
                                                uint64_t base_seed,
                                                const std::vector<std::vector<float>>& draft_logits = {});
    uint64_t total_draft_tokens() const;
    uint64_t total_accepted_tokens() const;
    double cumulative_acceptance_rate() const {
        return total_draft_tokens() == 0 ? 0.0 : (double)total_accepted_tokens() / (double)total_draft_tokens();
    }

   private:
    struct Impl;
    std::unique_ptr<Impl> impl_;
};

}  // namespace g4dense
