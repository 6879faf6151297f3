// Sampling parameters and host-side token draws with the reference's semantics
// (include/g4dense/sampling.hpp:9-27, src/sampling.cpp:56-169): greedy argmax with ties to the
// lowest index; otherwise top-k (at most 256) / top-p measured against the full-vocabulary
// softmax / temperature, drawn with xorshift64* from `seed`. Seeds per position follow seed_for.
#pragma once
#include <cstdint>
#include <vector>

#include "g4dense/device_context.hpp"

namespace g4dense {

struct SamplingParams {
    float temperature{0.0f};         // 0 = greedy
    float top_p{1.0f};               // 1 = no nucleus truncation
    int top_k{0};                    // 0 = no top-k truncation (shortlist of 256)
    float repetition_penalty{1.0f};  // 1 = disabled
    bool has_seed{false};
    uint64_t seed{0};
    bool is_greedy() const { return temperature <= 0.0f && repetition_penalty == 1.0f; }
};

// Throws std::invalid_argument for parameters the reference rejects.
G4DENSE_CXX_API void validate_sampling(const SamplingParams& p);
G4DENSE_CXX_API uint64_t splitmix64(uint64_t x);
G4DENSE_CXX_API uint64_t seed_for(const SamplingParams& p, int position);
G4DENSE_CXX_API void apply_repetition_penalty(float* logits, uint32_t vocab, const std::vector<uint32_t>& history,
                                              float penalty, float softcap);
G4DENSE_CXX_API uint32_t sample_token(const float* logits, uint32_t vocab, const SamplingParams& p, uint64_t seed);

}  // namespace g4dense
