// The drafter of speculative decoding, the reference's DraftRuntime
// (include/g4dense/draft_runtime.hpp:13-54, src/draft_runtime.cpp:46-103), as a fully resident
// model on a B200. generate_draft_tokens feeds the context tokens it has not seen yet, then runs
// k single-token steps, each drawing its token with sample_token and the per-step seed
// splitmix64(seed + step) (splitmix64(1337 + step) without a seed), and returns every step's
// full logits row. accept() tells it how much of the context survived verification.
#pragma once
#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include "g4dense/device_context.hpp"
#include "g4dense/sampling.hpp"

namespace g4dense {

struct DraftResult {
    std::vector<uint32_t> draft_tokens;
    std::vector<std::vector<float>> draft_logits;  // one full-vocabulary row per draft
    double draft_time_ms{0.0};
};

class G4DENSE_CXX_API DraftRuntime {
   public:
    DraftRuntime();
    ~DraftRuntime();
    // Loads a .g4dense drafter onto ctx's device (whole, never tensor-parallel). Throws
    // G4DenseFormatError-like std::runtime_error for a missing or malformed file.
    bool load_model(const std::string& model_path, std::shared_ptr<DeviceContext> ctx, int max_context = 4096);
    DraftResult generate_draft_tokens(const std::vector<uint32_t>& context_tokens, uint32_t k,
                                      const SamplingParams& sampling);
    // The reference sets its consumed count to the accepted context length; a fully accepted
    // round leaves the last draft unforwarded, so here the count is capped at what the drafter
    // actually forwarded and that token is fed on the next call.
    void accept(size_t accepted_context_length);
    void reset();
    bool is_loaded() const;
    uint32_t draft_k() const { return default_k_; }
    void set_draft_k(uint32_t k) { default_k_ = k; }

   private:
    struct Impl;
    std::unique_ptr<Impl> impl_;
    uint32_t default_k_{6};
};

}  // namespace g4dense
