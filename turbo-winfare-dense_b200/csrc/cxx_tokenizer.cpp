// The public C++ tokenizer classes (include/g4dense/tokenizer.hpp, detokenizer.hpp) over the
// engine's tokenizer (tokenizer.cpp). Errors surface as G4DenseFormatError, as the reference's do.
#include "g4dense/detokenizer.hpp"
#include "g4dense/tokenizer.hpp"
#include "tokenizer.h"
#include "tokenizer_impl.h"

namespace g4dense {

size_t utf8_repair(std::string_view in, bool flush_all, std::string& out) {
    return g4b::utf8_repair(in, flush_all, out);
}

namespace {
template <class F>
auto as_format_error(F&& f) -> decltype(f()) {
    try {
        return f();
    } catch (const G4DenseFormatError&) {
        throw;
    } catch (const std::runtime_error& e) {
        throw G4DenseFormatError(e.what());
    }
}
}  // namespace

Tokenizer::Tokenizer() : impl_(new Impl) {}
Tokenizer::~Tokenizer() = default;

bool Tokenizer::load_vocabulary(const std::string& vocab_file) {
    return as_format_error([&] {
        if (vocab_file.empty())
            throw G4DenseFormatError("Tokenizer::load_vocabulary called with no vocabulary path");
        impl_->t.load(vocab_file);
        return true;
    });
}

std::vector<uint32_t> Tokenizer::encode(const std::string& text, bool add_bos) const {
    return as_format_error([&] { return impl_->t.encode(text, add_bos); });
}
std::string Tokenizer::decode(const std::vector<uint32_t>& tokens, bool skip_special) const {
    return as_format_error([&] { return impl_->t.decode(tokens, skip_special); });
}
std::string Tokenizer::decode_single(uint32_t token, bool skip_special) const {
    return impl_->t.decode_single(token, skip_special);
}
bool Tokenizer::is_byte_fallback(uint32_t token, uint8_t& value) const { return impl_->t.byte_value(token, value); }
bool Tokenizer::is_special_token(uint32_t token) const { return impl_->t.is_special(token); }

std::string Tokenizer::apply_chat_template(const std::vector<ChatMessage>& messages) const {
    std::vector<g4b::Tokenizer::Message> m;
    m.reserve(messages.size());
    for (const auto& x : messages) m.push_back({x.role, x.content});
    return as_format_error([&] { return impl_->t.chat_template(m); });
}

uint32_t Tokenizer::bos_id() const { return impl_->t.bos(); }
uint32_t Tokenizer::eos_id() const { return impl_->t.eos(); }
uint32_t Tokenizer::pad_id() const { return impl_->t.pad(); }
uint32_t Tokenizer::unk_id() const { return impl_->t.unk(); }
uint32_t Tokenizer::end_of_turn_id() const { return impl_->t.end_of_turn(); }
uint32_t Tokenizer::vocab_size() const { return impl_->t.vocab_size(); }
bool Tokenizer::is_loaded() const { return impl_->t.loaded(); }

void Tokenizer::set_architecture(ModelArch arch) {
    impl_->t.set_arch(arch == ModelArch::MUSE_GLIMMER ? g4b::Tokenizer::Arch::MuseGlimmer
                                                      : g4b::Tokenizer::Arch::Gemma4);
}
ModelArch Tokenizer::architecture() const {
    return impl_->t.arch() == g4b::Tokenizer::Arch::MuseGlimmer ? ModelArch::MUSE_GLIMMER : ModelArch::GEMMA4;
}
const std::vector<uint32_t>& Tokenizer::stop_token_ids() const { return impl_->t.stop_ids(); }

struct IncrementalDetokenizer::Impl {
    Impl(const g4b::Tokenizer& t, bool skip) : d(t, skip) {}
    g4b::IncrementalDetokenizer d;
};

IncrementalDetokenizer::IncrementalDetokenizer(const Tokenizer& tok, bool skip_special)
    : impl_(new Impl(tok.impl_->t, skip_special)) {}
IncrementalDetokenizer::~IncrementalDetokenizer() = default;
std::string IncrementalDetokenizer::push(uint32_t token) { return impl_->d.push(token); }
std::string IncrementalDetokenizer::finish() { return impl_->d.finish(); }
void IncrementalDetokenizer::reset() { impl_->d.reset(); }

struct StreamingStopMatcher::Impl {
    g4b::StreamingStopMatcher m;
};

StreamingStopMatcher::StreamingStopMatcher() : impl_(new Impl) {}
StreamingStopMatcher::StreamingStopMatcher(std::vector<std::string> stops) : impl_(new Impl{g4b::StreamingStopMatcher(std::move(stops))}) {}
StreamingStopMatcher::~StreamingStopMatcher() = default;
StreamingStopMatcher::StreamingStopMatcher(const StreamingStopMatcher& o) : impl_(new Impl(*o.impl_)) {}
StreamingStopMatcher& StreamingStopMatcher::operator=(const StreamingStopMatcher& o) {
    if (this != &o) *impl_ = *o.impl_;
    return *this;
}
std::string StreamingStopMatcher::push(std::string_view text) { return impl_->m.push(text); }
std::string StreamingStopMatcher::finish() { return impl_->m.finish(); }
bool StreamingStopMatcher::stopped() const { return impl_->m.stopped(); }
const std::string& StreamingStopMatcher::matched() const { return impl_->m.matched(); }
bool StreamingStopMatcher::empty() const { return impl_->m.empty(); }

}  // namespace g4dense
