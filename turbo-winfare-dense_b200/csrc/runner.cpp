#include "runner.h"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <sstream>
#include <stdexcept>

namespace g4b {

namespace {
double now_ms() {
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

// Config-3 oracle drafter: the proposal for history index n replays the target's stream, or,
// with probability `rate` (a seeded coin per index), a different id.
uint32_t replay_propose(const std::vector<uint32_t>& stream, size_t n_prompt, size_t hist_index, double rate,
                        uint64_t seed, uint32_t vocab) {
    const long long i = (long long)hist_index - (long long)n_prompt;
    const uint32_t truth = (i >= 0 && i < (long long)stream.size()) ? stream[(size_t)i] : 0u;
    const uint64_t h = splitmix64(seed + (uint64_t)hist_index);
    const double u = (double)(h >> 11) * (1.0 / 9007199254740992.0);
    if (u < rate) return (uint32_t)((truth + 1u + (uint32_t)(splitmix64(h) % (vocab - 1))) % vocab);
    return truth;
}
// Rows of the next prefill pass over `remaining` prompt positions: whole tensor-core chunks
// (max_rows = 128) while more than kPrefillMinRows remain; a shorter tail runs as verify passes
// of up to 16 rows, which cost less than a mostly empty tensor-core chunk.
constexpr size_t kPrefillMinRows = 48;
int next_chunk(size_t remaining, int max_rows) {
    if (max_rows > kBatchRows && remaining > kPrefillMinRows) return (int)std::min<size_t>(remaining, max_rows);
    return (int)std::min<size_t>(remaining, kBatchRows);
}
}  // namespace

void DraftRuntime::catch_up(const std::vector<uint32_t>& ctx) {
    if (consumed_ > ctx.size()) consumed_ = 0;
    while (consumed_ + 1 < ctx.size()) {
        const int m = next_chunk(ctx.size() - 1 - consumed_, model_->max_rows());
        model_->run_plain(m, (int)consumed_, ctx.data() + consumed_, false);
        consumed_ += m;
    }
}

void Engine::order(cudaStream_t from, cudaStream_t to) {
    if (from == to) return;
    if (!order_ev_[0])
        for (auto& e : order_ev_) cuda_check(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "event");
    cudaEvent_t e = order_ev_[order_i_ ^= 1];  // alternate: a recorded event is reused one edge later
    cuda_check(cudaEventRecord(e, from), "event record");
    cuda_check(cudaStreamWaitEvent(to, e, 0), "stream wait");
}

void Engine::forward_batch(const uint32_t* ids, uint32_t batch, uint32_t base, float* out_logits, bool all_positions) {
    // 1..16 rows run the verify pass (every row's logits available); 17..max_rows() run a
    // tensor-core prefill chunk, which ranks only its last row.
    if (batch < 1 || batch > (uint32_t)target_->max_rows())
        throw std::invalid_argument("forward_batch: batch must be 1.." + std::to_string(target_->max_rows()));
    if (batch > (uint32_t)kBatchRows && out_logits && all_positions)
        throw std::invalid_argument("forward_batch: a batch of more than 16 rows returns the last row's logits only");
    if (base + batch > (uint32_t)target_->max_context()) throw std::invalid_argument("forward_batch: context exceeds max_context");
    target_->run_plain((int)batch, (int)base, ids, out_logits != nullptr);
    if (out_logits) {
        const int row0 = all_positions ? 0 : DeviceModel::result_row((int)batch);
        target_->logits_to_host(row0, all_positions ? (int)batch : 1, out_logits);
    }
    cuda_check(cudaStreamSynchronize(target_->stream()), "forward_batch");
}

// Prefill in chunks of up to 128 positions on the tensor cores, the tail in 16-row verify
// passes (the reference chunks by 8, src/runner.cpp:2129-2133; batched rows equal sequential
// positions, so the chunk width does not change results). Returns the greedy next token; for
// sampled decoding fills *last_logits instead.
uint32_t Engine::prefill(const std::vector<uint32_t>& toks, const GenerationOptions& opt, std::vector<float>* last) {
    const bool greedy = opt.sampling.is_greedy();
    const size_t n = toks.size();
    int m_last = 1;
    for (size_t i = 0; i < n;) {
        const int m = next_chunk(n - i, target_->max_rows());
        const bool is_last = i + m == n;
        target_->run_plain(m, (int)i, toks.data() + i, is_last && !greedy);
        m_last = m;
        i += m;
    }
    const HeadResult r = target_->fetch_result();
    const int row = DeviceModel::result_row(m_last);
    last_row_ = row;
    if (!greedy && last) {
        last->resize(target_->header().vocab_size);
        target_->logits_to_host(row, 1, last->data());
    }
    return r.argmax[row];
}

std::vector<uint32_t> Engine::generate(const std::vector<uint32_t>& prompt, const GenerationOptions& opt,
                                       const TokenCallback& on_token, const std::atomic<bool>* cancel) {
    stats_ = GenStats{};
    const double t0 = now_ms();
    validate_sampling(opt.sampling);
    const SamplingParams& sp = opt.sampling;
    const bool greedy = sp.is_greedy();
    DeviceModel& T = *target_;
    const uint32_t V = T.header().vocab_size;
    std::vector<uint32_t> history;
    for (uint32_t t : prompt) {
        if (t >= V) {
            // src/runner.cpp:2099-2109: small vocabularies wrap, large ones reject.
            if (V <= 4096) t %= V;
            else throw std::invalid_argument("token id " + std::to_string(t) + " exceeds model vocab size " + std::to_string(V));
        }
        history.push_back(t);
    }
    if (history.empty()) throw std::invalid_argument("generate: prompt is empty");
    if (history.size() + (size_t)opt.max_tokens + 16 > (size_t)T.max_context())
        throw std::invalid_argument("generate: prompt + max_tokens exceeds the KV capacity (max_context)");
    if (opt.max_tokens <= 0) return {};

    std::vector<uint32_t> out;
    std::vector<float> logits;
    const uint64_t l0 = T.launches() + (draft_ ? draft_->model().launches() : 0);
    const uint64_t h0 = T.h2d_bytes() + (draft_ ? draft_->model().h2d_bytes() : 0);
    const uint64_t d0 = T.d2h_bytes() + (draft_ ? draft_->model().d2h_bytes() : 0);
    const bool spec = opt.speculative_enabled && has_drafter() && opt.draft_k > 0;
    stats_.draft_k = spec ? std::min<uint32_t>(opt.draft_k, kMaxDraftWidth) : 0;
    if (spec && draft_) {
        // The drafter's pass over the prompt is prefill work: queue it on the drafter's stream
        // first so it runs alongside the target's prefill.
        draft_->reset();
        draft_->catch_up(history);
    }
    // The device draw needs the whole vocabulary on one GPU; tensor-parallel ranks gather the
    // logits rows and draw on the host.
    const bool dev_sample = !greedy && !spec && opt.device_sampling && T.options().tp == 1;
    const uint32_t first = prefill(history, opt, dev_sample ? nullptr : &logits);
    if (spec && draft_) order(draft_->model().stream(), T.stream());  // decode starts after both prefills
    mtp_row_ = last_row_;  // the MTP drafter's first round starts from the prompt's last hidden state
    stats_.h2d_bytes += history.size() * sizeof(uint32_t);
    stats_.ttft_ms = now_ms() - t0;
    const double t_decode = now_ms();
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    cuda_check(cudaEventCreate(&ev0), "event");
    cuda_check(cudaEventCreate(&ev1), "event");
    cuda_check(cudaEventRecord(ev0, T.stream()), "event");

    int emitted = 0;
    auto emit = [&](uint32_t t) -> bool {
        out.push_back(t);
        ++stats_.emitted;
        if (on_token && !on_token(t)) {
            stats_.stop_reason = 2;
            return false;
        }
        if ((opt.stop_token >= 0 && (int64_t)t == opt.stop_token) ||
            std::find(opt.stop_tokens.begin(), opt.stop_tokens.end(), t) != opt.stop_tokens.end()) {
            stats_.stop_reason = 1;
            return false;
        }
        return true;
    };
    if (spec) {
        // Two kinds of drafter: a separate model with its own KV (DraftRuntime) or the MTP
        // assistant (src/mtp_runner.cpp), which reads the target's KV and hidden state and runs
        // on the target's stream.
        // Under tensor parallelism only rank 0 holds the drafter (Dmp is null elsewhere): its
        // drafts reach the other ranks by broadcast before each verify pass.
        DraftRuntime* Dp = draft_.get();
        DeviceModel* Mt = mtp_.get();
        DeviceModel* Dmp = Dp ? &Dp->model() : Mt;
        if (Dmp && Dmp->header().vocab_size != V)
            throw std::invalid_argument("drafter vocabulary differs from the target's");
        const bool tp_multi = T.options().tp > 1;
        const bool evaluates = !tp_multi || T.options().rank == 0;
        const uint32_t K = std::min<uint32_t>(opt.draft_k, kMaxDraftWidth);
        uint32_t drafted_total = 0, accepted_total = 0;
        bool drafting = true;
        uint32_t pending = greedy ? first : sample_token(logits.data(), V, sp, seed_for(sp, (int)history.size() - 1));
        history.push_back(pending);
        ++emitted;
        bool stop = !emit(pending);
        std::vector<float> verify, dl;
        while (!stop && emitted < opt.max_tokens) {
            if (cancel && cancel->load()) {
                stats_.stop_reason = 3;
                break;
            }
            if (!drafting) {
                // Gated: one target pass per token (src/runner.cpp:2219-2237).
                T.run_plain(1, (int)history.size() - 1, &pending, !greedy);
                mtp_row_ = 0;
                const HeadResult r = T.fetch_result();
                uint32_t nx = r.argmax[0];
                if (!greedy) {
                    verify.resize(V);
                    T.logits_to_host(0, 1, verify.data());
                    nx = sample_token(verify.data(), V, sp, seed_for(sp, (int)history.size()));
                }
                history.push_back(nx);
                ++emitted;
                ++stats_.gated_steps;
                pending = nx;
                if (!emit(nx)) break;
                continue;
            }
            if (K < 2) break;  // K-1 = 0 drafts: the reference's round loop ends here
            const double tr0 = now_ms();
            const size_t len = history.size();
            // Greedy: context the drafter has not seen yet (one token after a fully accepted
            // round) rides in the first drafting pass together with the pending token, so that
            // round needs no separate catch-up pass. Batched rows equal sequential positions.
            size_t unseen = 0;
            if (Dp && greedy) {
                if (Dp->consumed() > len - 1) Dp->set_consumed(0);
                unseen = len - 1 - Dp->consumed();
                if (unseen + 1 > (size_t)kBatchRows) {
                    Dp->catch_up(history);
                    unseen = 0;
                }
            } else if (Dp) {
                Dp->catch_up(history);
            }
            std::vector<uint32_t> emitted_now;
            uint32_t n_acc = 0;
            if (greedy && Mt) {
                // MTP round: the drafter's steps chain their tokens into the verify pass's step
                // parameters on the device. Its query sits at the pending token's position and
                // attends the keys the target has processed (positions up to len - 2).
                StepParams tp{}, mp{};
                tp.base_pos = (int)len - 1;
                tp.tokens[0] = pending;
                mp.base_pos = (int)len - 2;
                mp.tokens[0] = pending;
                mp.aux = mtp_row_;
                const bool replay = !opt.replay.empty();
                T.push_params(0, tp);
                Mt->push_params(1, mp, 1);
                uint32_t* chain = replay ? Mt->chain_dev() : T.step_params(0)->tokens + 1;
                for (uint32_t s = 0; s + 1 < K; ++s)
                    Mt->enqueue(1, s == 0 ? PassKind::MtpFirst : PassKind::MtpNext, false, chain);
                if (replay) {
                    for (uint32_t s = 0; s + 1 < K; ++s)
                        tp.tokens[s + 1] = replay_propose(opt.replay, prompt.size(), len + s, opt.mismatch_rate,
                                                          opt.mismatch_seed, V);
                    T.push_params(0, tp);
                }
                T.enqueue((int)K, PassKind::Plain, false, nullptr);
                const HeadResult r = T.fetch_result();
                n_acc = (uint32_t)r.n_accepted;
                emitted_now.assign(r.tokens, r.tokens + r.n_emit);
            } else if (greedy) {
                StepParams tp{}, dp{};
                tp.base_pos = (int)len - 1;
                tp.tokens[0] = pending;
                dp.base_pos = (int)(len - 1 - unseen);
                for (size_t i = 0; i < unseen; ++i) dp.tokens[i] = history[len - 1 - unseen + i];
                dp.tokens[unseen] = pending;
                const bool replay = !opt.replay.empty();
                T.push_params(0, tp);
                if (Dp) {
                    // The drafter's steps write their tokens into the target's step parameters:
                    // after the target's parameter copy, and before the verify pass reads them.
                    DeviceModel& Dm = *Dmp;
                    order(T.stream(), Dm.stream());
                    Dm.push_params(1, dp, (int)unseen + 1);
                    uint32_t* chain = replay ? Dm.chain_dev() : T.step_params(0)->tokens + 1;
                    for (uint32_t s = 0; s + 1 < K; ++s)
                        Dm.enqueue(s == 0 ? (int)unseen + 1 : 1, PassKind::DraftStep, false, chain);
                    Dp->set_consumed(len - 1);
                }
                if (replay) {
                    for (uint32_t s = 0; s + 1 < K; ++s)
                        tp.tokens[s + 1] = replay_propose(opt.replay, prompt.size(), len + s, opt.mismatch_rate,
                                                          opt.mismatch_seed, V);
                    T.push_params(0, tp);
                }
                if (Dp) order(Dmp->stream(), T.stream());  // replay too: the verify waits for the drafts
                T.bcast_step_tokens((int)K - 1);           // rank 0's drafts into every rank's pass
                T.enqueue((int)K, PassKind::Plain, false, nullptr);
                const HeadResult r = T.fetch_result();
                n_acc = (uint32_t)r.n_accepted;
                emitted_now.assign(r.tokens, r.tokens + r.n_emit);
            } else {
                // Sampled: the reference's host RNG streams decide drafts and acceptance.
                std::vector<uint32_t> drafts;
                std::vector<std::vector<float>> draft_logits;
                uint32_t cur = pending;
                int pos = (int)len - 1;
                for (uint32_t s = 0; Dmp && s + 1 < K; ++s) {
                    DeviceModel& Dm = *Dmp;
                    if (Mt) {
                        StepParams mp{};
                        mp.base_pos = (int)len - 2;
                        mp.tokens[0] = cur;
                        mp.aux = mtp_row_;
                        Mt->push_params(1, mp, 1);
                        Mt->enqueue(1, s == 0 ? PassKind::MtpFirst : PassKind::MtpNext, true, nullptr);
                    } else {
                        Dm.run_plain(1, pos++, &cur, true);
                    }
                    dl.resize(V);
                    cuda_check(cudaMemcpyAsync(dl.data(), Dm.logits_dev(), V * 4, cudaMemcpyDeviceToHost, Dm.stream()),
                               "logits");
                    cuda_check(cudaStreamSynchronize(Dm.stream()), "sync");
                    const uint64_t ss = splitmix64(sp.has_seed ? (sp.seed + s) : (1337 + s));
                    const uint32_t cand = sample_token(dl.data(), V, sp, ss);
                    drafts.push_back(cand);
                    draft_logits.push_back(dl);
                    cur = cand;
                }
                drafts.resize(K - 1);
                T.bcast_host_u32(drafts.data(), (int)K - 1);  // rank 0's drafts to every rank
                std::vector<uint32_t> batch = {pending};
                batch.insert(batch.end(), drafts.begin(), drafts.end());
                T.run_plain((int)K, (int)len - 1, batch.data(), true);
                verify.resize((size_t)K * V);
                T.logits_to_host(0, (int)K, verify.data());
                // The ratio test needs the drafter's logits, so rank 0 decides and broadcasts
                // {accepted, count, tokens...}.
                std::vector<uint32_t> res(K + 2, 0u);
                if (evaluates) {
                    std::vector<const float*> per_pos;
                    for (uint32_t i = 0; i < K; ++i) per_pos.push_back(verify.data() + (size_t)i * V);
                    const SpeculativeEvaluation ev =
                        speculator_.evaluate_verification(drafts, per_pos, V, sp, seed_for(sp, (int)len), draft_logits);
                    res[0] = ev.num_accepted;
                    res[1] = (uint32_t)ev.accepted_tokens.size();
                    std::copy(ev.accepted_tokens.begin(), ev.accepted_tokens.end(), res.begin() + 2);
                }
                if (tp_multi) T.bcast_host_u32(res.data(), (int)K + 2);
                n_acc = res[0];
                emitted_now.assign(res.begin() + 2, res.begin() + 2 + std::min<uint32_t>(res[1], K));
            }
            const size_t forwarded = (len - 1) + (K - 1);
            int this_emit = 0;
            for (uint32_t t : emitted_now) {
                if (emitted >= opt.max_tokens) {
                    stop = true;
                    break;
                }
                history.push_back(t);
                ++emitted;
                ++this_emit;
                pending = t;
                if (!emit(t)) {
                    stop = true;
                    break;
                }
            }
            if (Dp) Dp->accept(history.size() - 1, forwarded);
            mtp_row_ = (int)n_acc;  // the verify row whose logits gave the round's last token
            ++stats_.rounds;
            stats_.drafted += K - 1;
            stats_.accepted += n_acc;
            stats_.round_info.push_back((int)(K - 1));
            stats_.round_info.push_back((int)n_acc);
            stats_.round_info.push_back(this_emit);
            stats_.verify_ms += now_ms() - tr0;
            drafted_total += K - 1;
            accepted_total += n_acc;
            if (drafting && opt.gate_window >= 0 && drafted_total >= (uint32_t)opt.gate_window &&
                (double)accepted_total / drafted_total < opt.gate_min_accept) {
                drafting = false;
                stats_.gated = true;
            }
        }
    } else {
        // Non-speculative loop (src/runner.cpp:2314-2344).
        uint32_t next_greedy = first;
        for (int step = 0; step < opt.max_tokens; ++step) {
            if (cancel && cancel->load()) {
                stats_.stop_reason = 3;
                break;
            }
            const int pos = (int)history.size() - 1;
            uint32_t nx = next_greedy;
            if (dev_sample) {
                if (step == 0 && sp.repetition_penalty != 1.0f) T.rep_reset(history.data(), (int)history.size());
                nx = T.sample_device(last_row_, sp.temperature, sp.top_p, sp.top_k, seed_for(sp, pos),
                                     sp.repetition_penalty);
            } else if (!greedy) {
                if (sp.repetition_penalty != 1.0f)
                    apply_repetition_penalty(logits.data(), V, history, sp.repetition_penalty,
                                             T.header().final_logit_softcapping);
                nx = sample_token(logits.data(), V, sp, seed_for(sp, pos));
            }
            history.push_back(nx);
            ++emitted;
            if (!emit(nx)) break;
            if (emitted >= opt.max_tokens) break;
            T.run_plain(1, (int)history.size() - 1, &nx, !greedy);
            last_row_ = 0;
            if (dev_sample) continue;  // the next draw reads the logits on the device
            const HeadResult r = T.fetch_result();
            next_greedy = r.argmax[0];
            if (!greedy) {
                logits.resize(V);
                T.logits_to_host(0, 1, logits.data());
            }
        }
    }
    cuda_check(cudaEventRecord(ev1, T.stream()), "event");
    cuda_check(cudaEventSynchronize(ev1), "event");
    float dms = 0.f;
    cuda_check(cudaEventElapsedTime(&dms, ev0, ev1), "event");
    cudaEventDestroy(ev0);
    cudaEventDestroy(ev1);
    stats_.decode_gpu_ms = dms;
    T.check_device_error();
    stats_.total_ms = now_ms() - t0;
    stats_.decode_ms = now_ms() - t_decode;
    stats_.launches = T.launches() + (draft_ ? draft_->model().launches() : 0) - l0;
    stats_.h2d_bytes += T.h2d_bytes() + (draft_ ? draft_->model().h2d_bytes() : 0) - h0;
    stats_.d2h_bytes += T.d2h_bytes() + (draft_ ? draft_->model().d2h_bytes() : 0) - d0 + out.size() * sizeof(uint32_t);
    stats_.context_tokens = history.size();
    return out;
}

std::string Engine::telemetry_json() const {
    std::ostringstream ss;
    ss.setf(std::ios::fixed);
    ss.precision(2);
    const GenStats& s = stats_;
    const double tps = s.decode_ms > 0 ? (double)s.emitted / (s.decode_ms / 1000.0) : 0.0;
    const double rate = s.drafted ? 100.0 * (double)s.accepted / (double)s.drafted : 0.0;
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceProp prop{};
    cudaGetDeviceProperties(&prop, dev);
    const G4DenseHeader& h = target_->header();
    ss << "{\n";
    ss << "  \"tps\": " << tps << ",\n";
    ss << "  \"ttft_ms\": " << s.ttft_ms << ",\n";
    ss << "  \"speculative_acceptance_rate\": " << rate << ",\n";
    ss << "  \"max_context\": " << target_->max_context() << ",\n";
    ss << "  \"gpu_name\": \"" << prop.name << "\",\n";
    ss << "  \"has_draft\": " << (draft_ || mtp_ ? "true" : "false") << ",\n";
    ss << "  \"speculative_drafted\": " << s.drafted << ",\n";
    ss << "  \"speculative_accepted\": " << s.accepted << ",\n";
    ss << "  \"drafting_gated\": " << (s.gated ? "true" : "false") << ",\n";
    ss << "  \"total_tokens_generated\": " << s.emitted << ",\n";
    ss << "  \"kv_cache_mb\": " << (double)target_->kv_bytes() / 1048576.0 << ",\n";
    ss << "  \"layer_mb\": " << (double)target_->weight_bytes() / 1048576.0 / std::max(1u, h.num_layers) << ",\n";
    ss << "  \"total_layers\": " << h.num_layers << ",\n";
    ss << "  \"pinned_layers\": " << h.num_layers << ",\n";  // every layer is resident in HBM
    ss << "  \"streamed_layers\": 0,\n";
    ss << "  \"lm_head_mb\": "
       << ((double)h.vocab_size * h.d_model / 2 + (double)h.vocab_size * (h.d_model / 64) * 4) / 1048576.0 << ",\n";
    ss << "  \"draft_k\": " << s.draft_k << ",\n";
    ss << "  \"context_tokens\": " << s.context_tokens << ",\n";
    ss << "  \"speculative_rounds\": " << s.rounds << ",\n";
    ss << "  \"gated_steps\": " << s.gated_steps << ",\n";
    ss << "  \"tensor_parallel\": " << target_->options().tp << ",\n";
    ss << "  \"breakdown\": {\n";
    ss << "    \"decode_ms\": " << s.decode_ms << ",\n";
    ss << "    \"round_ms\": " << s.verify_ms << "\n";
    ss << "  }\n";
    ss << "}\n";
    return ss.str();
}

}  // namespace g4b
