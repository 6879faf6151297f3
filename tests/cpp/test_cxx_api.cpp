// Links libg4dense_b200.so through the public C++ headers (include/g4dense/*.hpp), the way the
// reference's own C++ callers use ForwardRunner / DraftRuntime / SpeculativeCoordinator.
//
//   test_cxx_api cpu
//       known answers that need no GPU: splitmix64 (the reference's tests/test_sampling.cpp:118-121),
//       the greedy tie rule (tests/test_sampling.cpp:139-149), greedy acceptance
//       (tests/test_speculative.cpp:29-77), and the load errors of a missing container.
//   test_cxx_api gpu <target.g4dense> <draft.g4dense> <prompt ids, comma-separated> <n>
//       prints one JSON object: the target's logits argmax per position (forward_batch of all
//       positions vs forward_single_token), greedy speculative generate_tokens with its round
//       records, the plain greedy stream, and DraftRuntime drafts for the prompt. The pytest
//       wrapper compares them with the CPU oracle.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <sstream>
#include <string>
#include <vector>

#include "g4dense/draft_runtime.hpp"
#include "g4dense/runner.hpp"
#include "g4dense/sampling.hpp"
#include "g4dense/speculator.hpp"

using namespace g4dense;

static int failures = 0;
#define CHECK(c)                                                         \
    do {                                                                 \
        if (!(c)) {                                                      \
            std::fprintf(stderr, "CHECK failed: %s (line %d)\n", #c, __LINE__); \
            ++failures;                                                  \
        }                                                                \
    } while (0)

static std::string join(const std::vector<uint32_t>& v) {
    std::ostringstream s;
    for (size_t i = 0; i < v.size(); ++i) s << (i ? "," : "") << v[i];
    return s.str();
}

static int run_cpu() {
    CHECK(splitmix64(0) == 0xE220A8397B1DCDAFull);
    CHECK(splitmix64(1) == 0x910A2DEC89025CC1ull);
    CHECK(splitmix64(2) == 0x975835DE1C9756CEull);
    CHECK(splitmix64(3) == 0x1D0B14E4DB018FEDull);
    const float tie[5] = {1.f, 5.f, 3.f, 5.f, 2.f};
    CHECK(sample_token(tie, 5, SamplingParams{}, 1) == 1);
    SamplingParams bad;
    bad.top_p = 0.f;
    bool threw = false;
    try {
        validate_sampling(bad);
    } catch (const std::invalid_argument&) {
        threw = true;
    }
    CHECK(threw);

    // Greedy acceptance: one-hot target rows at 42, 100, 200, 300, 400.
    std::vector<std::vector<float>> rows(5, std::vector<float>(1024, 0.f));
    const uint32_t hot[5] = {42, 100, 200, 300, 400};
    for (int i = 0; i < 5; ++i) rows[i][hot[i]] = 10.f;
    std::vector<const float*> per_pos;
    for (auto& r : rows) per_pos.push_back(r.data());
    SpeculativeCoordinator sc;
    SpeculativeEvaluation e = sc.evaluate_verification({42, 100, 200, 300}, per_pos, 1024, SamplingParams{}, 12345);
    CHECK(e.num_accepted == 4 && e.accepted_tokens == (std::vector<uint32_t>{42, 100, 200, 300, 400}));
    e = sc.evaluate_verification({42, 100, 999, 300}, per_pos, 1024, SamplingParams{}, 12345);
    CHECK(e.num_accepted == 2 && e.accepted_tokens == (std::vector<uint32_t>{42, 100, 200}));
    e = sc.evaluate_verification({999, 100}, std::vector<const float*>(per_pos.begin(), per_pos.begin() + 3), 1024,
                                 SamplingParams{}, 12345);
    CHECK(e.num_accepted == 0 && e.accepted_tokens == (std::vector<uint32_t>{42}));
    CHECK(sc.total_draft_tokens() == 10 && sc.total_accepted_tokens() == 6);

    // A missing container fails loudly at initialize(), as the reference's constructor does.
    threw = false;
    try {
        std::shared_ptr<DeviceContext> ctx;  // no device needed to reach the argument check
        ForwardRunner r(ctx, "missing.g4dense");
    } catch (const std::invalid_argument&) {
        threw = true;
    }
    CHECK(threw);
    DraftRuntime d;
    CHECK(!d.is_loaded());
    CHECK(d.generate_draft_tokens({1, 2, 3}, 4, SamplingParams{}).draft_tokens.empty());
    std::printf("{\"cpu_failures\": %d}\n", failures);
    return failures ? 1 : 0;
}

static int run_gpu(const char* target, const char* draft, const char* prompt_csv, int n) {
    std::vector<uint32_t> prompt;
    for (const char* p = prompt_csv; *p;) {
        prompt.push_back((uint32_t)std::strtoul(p, (char**)&p, 10));
        if (*p == ',') ++p;
    }
    auto ctx = DeviceContext::create(0);
    ForwardRunner runner(ctx, target);
    runner.set_max_context(1024);
    runner.initialize();
    const uint32_t V = runner.vocab_size();

    // forward_batch over the first 8 prompt positions vs forward_single_token position by position.
    const uint32_t B = 8;
    std::vector<float> batched(B * V), single(V);
    runner.forward_batch(prompt.data(), B, 0, batched.data(), true);
    runner.reset_kv_cache();
    std::vector<uint32_t> am_batched, am_single;
    double worst = 0.0;
    for (uint32_t i = 0; i < B; ++i) {
        runner.forward_single_token(prompt[i], i, single.data());
        uint32_t a = 0, b = 0;
        for (uint32_t v = 1; v < V; ++v) {
            if (batched[i * V + v] > batched[i * V + a]) a = v;
            if (single[v] > single[b]) b = v;
            worst = std::fmax(worst, std::fabs(batched[i * V + v] - single[v]));
        }
        am_batched.push_back(a);
        am_single.push_back(b);
    }

    GenerationOptions o;
    o.max_tokens = n;
    o.use_chat_template = false;
    const std::vector<uint32_t> plain = runner.generate_tokens(prompt, o);
    runner.load_draft_model(draft);
    CHECK(runner.has_draft_model());
    o.speculative_enabled = true;
    o.draft_k = 5;
    int streamed = 0;
    const std::vector<uint32_t> spec = runner.generate_tokens(prompt, o, [&](uint32_t, const std::string&) {
        ++streamed;
        return true;
    });
    std::ostringstream rounds;
    for (const RoundRecord& r : runner.last_rounds())
        rounds << (rounds.tellp() > 0 ? "," : "") << "[" << r.drafted << "," << r.accepted << "," << r.emitted << "]";

    // The text entry point refuses without a tokenizer.
    bool threw = false;
    try {
        runner.generate("hello", o, nullptr);
    } catch (const std::runtime_error&) {
        threw = true;
    }
    CHECK(threw);

    // DraftRuntime on its own: 4 greedy drafts continuing the prompt, then accept 2 of them and
    // draft again from the kept context.
    DraftRuntime dr;
    dr.load_model(draft, ctx, 1024);
    const DraftResult d1 = dr.generate_draft_tokens(prompt, 4, SamplingParams{});
    CHECK(d1.draft_tokens.size() == 4 && d1.draft_logits.size() == 4 && d1.draft_logits[0].size() == V);
    std::vector<uint32_t> kept = prompt;
    kept.insert(kept.end(), d1.draft_tokens.begin(), d1.draft_tokens.begin() + 2);
    dr.accept(kept.size());
    const DraftResult d2 = dr.generate_draft_tokens(kept, 3, SamplingParams{});

    std::printf(
        "{\"failures\": %d, \"argmax_batched\": [%s], \"argmax_single\": [%s], \"batched_vs_single_max_diff\": %.3e, "
        "\"plain\": [%s], \"spec\": [%s], \"spec_streamed\": %d, \"rounds\": [%s], \"draft1\": [%s], "
        "\"draft2\": [%s]}\n",
        failures, join(am_batched).c_str(), join(am_single).c_str(), worst, join(plain).c_str(), join(spec).c_str(),
        streamed, rounds.str().c_str(), join(d1.draft_tokens).c_str(), join(d2.draft_tokens).c_str());
    return failures ? 1 : 0;
}

int main(int argc, char** argv) {
    try {
        if (argc >= 2 && std::strcmp(argv[1], "cpu") == 0) return run_cpu();
        if (argc >= 6 && std::strcmp(argv[1], "gpu") == 0) return run_gpu(argv[2], argv[3], argv[4], std::atoi(argv[5]));
    } catch (const std::exception& e) {
        std::fprintf(stderr, "exception: %s\n", e.what());
        return 2;
    }
    std::fprintf(stderr, "usage: test_cxx_api cpu | gpu <target> <draft> <ids> <n>\n");
    return 2;
}
