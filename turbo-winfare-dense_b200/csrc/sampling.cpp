#include "sampling.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <numeric>
#include <random>
#include <stdexcept>
#include <string>

namespace g4b {

namespace {
constexpr int kMaxTopK = 256;  // src/sampling.cpp:215

// xorshift64* (src/sampling.cpp:218-228): one uniform per drawn token.
inline uint64_t next_random(uint64_t& s) {
    s ^= s >> 12;
    s ^= s << 25;
    s ^= s >> 27;
    return s * 0x2545F4914F6CDD1DULL;
}
inline float next_uniform(uint64_t& s) {
    return static_cast<float>((next_random(s) >> 40) & 0xFFFFFF) / 16777216.0f;
}

// compute_softmax (src/speculator.cpp:14-30)
void softmax_t(float* l, uint32_t n, float temp) {
    if (temp <= 0.0f) temp = 1.0f;
    float mx = -1e9f;
    for (uint32_t i = 0; i < n; ++i) {
        l[i] /= temp;
        if (l[i] > mx) mx = l[i];
    }
    float sum = 0.0f;
    for (uint32_t i = 0; i < n; ++i) {
        l[i] = std::exp(l[i] - mx);
        sum += l[i];
    }
    const float inv = 1.0f / (sum > 1e-12f ? sum : 1.0f);
    for (uint32_t i = 0; i < n; ++i) l[i] *= inv;
}
}  // namespace

void validate_sampling(const SamplingParams& p) {
    if (!std::isfinite(p.temperature) || p.temperature < 0.0f)
        throw std::invalid_argument("temperature must be finite and >= 0 (0 = greedy)");
    if (!std::isfinite(p.top_p) || p.top_p <= 0.0f || p.top_p > 1.0f) throw std::invalid_argument("top_p must be in (0, 1]");
    if (p.top_k < 0 || p.top_k > kMaxTopK)
        throw std::invalid_argument("top_k must be in 0.." + std::to_string(kMaxTopK) + " (0 disables it)");
    if (!std::isfinite(p.repetition_penalty) || p.repetition_penalty <= 0.0f)
        throw std::invalid_argument("repetition_penalty must be finite and > 0 (1 = disabled)");
    if (p.temperature > 0.0f && p.top_p < 1.0f && p.top_k == 0)
        throw std::invalid_argument("top_p < 1 with temperature > 0 requires top_k in 1.." + std::to_string(kMaxTopK) +
                                    "; full-vocabulary nucleus sampling is not implemented");
}

uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ULL;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ULL;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBULL;
    return x ^ (x >> 31);
}

uint64_t seed_for(const SamplingParams& p, int position) {
    const uint64_t base = p.has_seed ? p.seed + static_cast<uint64_t>(position)
                                     : (0x9E3779B97F4A7C15ULL ^ (static_cast<uint64_t>(position) * 0xD1B54A32D192ED03ULL));
    const uint64_t s = splitmix64(base);
    return s ? s : 0x9E3779B97F4A7C15ULL;
}

void apply_repetition_penalty(float* logits, uint32_t vocab, const std::vector<uint32_t>& history, float penalty,
                              float softcap) {
    if (penalty == 1.0f || history.empty()) return;
    const float limit = softcap > 0.0f ? softcap * 0.9999f : 0.0f;
    for (uint32_t id : history) {
        if (id >= vocab) continue;
        float v = logits[id];
        v = v > 0.0f ? v / penalty : v * penalty;
        if (limit > 0.0f) v = std::clamp(v, -limit, limit);
        logits[id] = v;
    }
}

uint32_t sample_token(const float* logits, uint32_t vocab, const SamplingParams& p, uint64_t seed) {
    if (vocab == 0) throw std::invalid_argument("sample_token: empty vocabulary");
    if (p.temperature <= 0.0f) {
        uint32_t best = 0;
        float bv = logits[0];
        for (uint32_t i = 1; i < vocab; ++i)
            if (logits[i] > bv) {
                bv = logits[i];
                best = i;
            }
        return best;
    }
    float mx = logits[0];
    for (uint32_t i = 1; i < vocab; ++i) mx = std::max(mx, logits[i]);
    double total = 0.0;
    for (uint32_t i = 0; i < vocab; ++i) total += std::exp(static_cast<double>(logits[i]) - mx);
    if (!(total > 0.0)) throw std::invalid_argument("sample_token: logit distribution is degenerate");
    const size_t want = p.top_k > 0 ? std::min<size_t>((size_t)p.top_k, vocab) : std::min<size_t>(kMaxTopK, vocab);
    std::vector<uint32_t> idx(vocab);
    std::iota(idx.begin(), idx.end(), 0u);
    auto by_desc = [&](uint32_t a, uint32_t b) {
        if (logits[a] != logits[b]) return logits[a] > logits[b];
        return a < b;
    };
    if (want < idx.size()) {
        std::nth_element(idx.begin(), idx.begin() + (ptrdiff_t)want, idx.end(), by_desc);
        idx.resize(want);
    }
    std::sort(idx.begin(), idx.end(), by_desc);
    size_t cut = idx.size();
    if (p.top_p < 1.0f) {
        double run = 0.0;
        for (size_t i = 0; i < idx.size(); ++i) {
            run += std::exp(static_cast<double>(logits[idx[i]]) - mx) / total;
            if (run >= static_cast<double>(p.top_p)) {
                cut = i + 1;
                break;
            }
        }
    }
    if (p.top_k > 0) cut = std::min(cut, (size_t)p.top_k);
    cut = std::max<size_t>(1, cut);
    std::vector<double> q(cut);
    double denom = 0.0;
    for (size_t i = 0; i < cut; ++i) {
        q[i] = std::exp((static_cast<double>(logits[idx[i]]) - mx) / p.temperature);
        denom += q[i];
    }
    uint64_t state = seed;
    const double r = static_cast<double>(next_uniform(state)) * denom;
    double acc = 0.0;
    for (size_t i = 0; i < cut; ++i) {
        acc += q[i];
        if (acc >= r) return idx[i];
    }
    return idx[cut - 1];
}

SpeculativeEvaluation SpeculativeCoordinator::evaluate_verification(
    const std::vector<uint32_t>& drafts, const std::vector<const float*>& target, uint32_t V,
    const SamplingParams& sp, uint64_t base_seed, const std::vector<std::vector<float>>& draft_logits) {
    SpeculativeEvaluation ev{};
    ev.total_drafted = (uint32_t)drafts.size();
    total_draft_ += ev.total_drafted;
    if (drafts.empty() || target.empty()) return ev;
    const size_t k = std::min(drafts.size(), target.size());
    size_t accepted = 0;
    for (size_t i = 0; i < k; ++i) {
        const uint32_t dt = drafts[i];
        const float* lg = target[i];
        const uint64_t step_seed = splitmix64(base_seed + i);
        const bool has_q = i < draft_logits.size() && !draft_logits[i].empty();
        if (sp.is_greedy() || !has_q) {
            const uint32_t tt = sample_token(lg, V, sp, step_seed);
            if (dt == tt) {
                ev.accepted_tokens.push_back(dt);
                ++accepted;
                continue;
            }
            ev.bonus_token = tt;
            ev.bonus_token_sampled = true;
            ev.accepted_tokens.push_back(tt);
            break;
        }
        // Rejection sampling against the draft distribution (src/speculator.cpp:71-122).
        std::vector<float> pt(lg, lg + V), qd(draft_logits[i]);
        softmax_t(pt.data(), V, sp.temperature);
        softmax_t(qd.data(), V, sp.temperature);
        const float pv = dt < V ? pt[dt] : 0.0f, qv = dt < V ? qd[dt] : 0.0f;
        const float r = qv > 1e-12f ? pv / qv : 1.0f;
        std::mt19937_64 rng(step_seed);
        std::uniform_real_distribution<float> ud(0.0f, 1.0f);
        const float u = ud(rng);
        if (u <= r) {
            ev.accepted_tokens.push_back(dt);
            ++accepted;
            continue;
        }
        float sum_diff = 0.0f;
        for (uint32_t v = 0; v < V; ++v) {
            const float dd = std::max(0.0f, pt[v] - qd[v]);
            qd[v] = dd;
            sum_diff += dd;
        }
        uint32_t corr = 0;
        if (sum_diff > 1e-9f) {
            const float rv = ud(rng) * sum_diff;
            float acc = 0.0f;
            for (uint32_t v = 0; v < V; ++v) {
                acc += qd[v];
                if (acc >= rv) {
                    corr = v;
                    break;
                }
            }
        } else {
            corr = sample_token(lg, V, sp, step_seed);
        }
        ev.bonus_token = corr;
        ev.bonus_token_sampled = true;
        ev.accepted_tokens.push_back(corr);
        break;
    }
    if (accepted == k && target.size() > k) {
        const uint32_t b = sample_token(target[k], V, sp, splitmix64(base_seed + k));
        ev.bonus_token = b;
        ev.bonus_token_sampled = true;
        ev.accepted_tokens.push_back(b);
    }
    ev.num_accepted = (uint32_t)accepted;
    total_accepted_ += ev.num_accepted;
    ev.acceptance_rate = ev.total_drafted ? (double)ev.num_accepted / ev.total_drafted : 0.0;
    return ev;
}

}  // namespace g4b
