// The reference's Tokenizer (include/g4dense/tokenizer.hpp:1-105 of the reference; behaviour of
// src/tokenizer.cpp): Gemma-4 tokenizer.json BPE with byte fallback, the chat template, special
// and stop ids. Same class, method names, argument meanings and exceptions; the implementation is
// this library's (a heap-driven BPE with the reference's merge order).
#pragma once
#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>
#include <string_view>
#include <vector>

#include "g4dense/device_context.hpp"

namespace g4dense {

// include/g4dense/format.hpp:114-117 and :249-253 of the reference.
enum class ModelArch : uint32_t { GEMMA4 = 0, MUSE_GLIMMER = 1 };

class G4DenseFormatError : public std::runtime_error {
   public:
    explicit G4DenseFormatError(const std::string& message) : std::runtime_error(message) {}
};

// Appends the valid UTF-8 prefix of `in` to `out` (U+FFFD for bytes that cannot form a
// character) and returns the bytes of `in` consumed; an incomplete tail is held back unless
// flush_all, when it becomes one U+FFFD.
G4DENSE_CXX_API size_t utf8_repair(std::string_view in, bool flush_all, std::string& out);

class G4DENSE_CXX_API Tokenizer {
   public:
    Tokenizer();
    ~Tokenizer();
    Tokenizer(const Tokenizer&) = delete;
    Tokenizer& operator=(const Tokenizer&) = delete;

    // Reads a Hugging Face tokenizer.json. Throws G4DenseFormatError for an empty path (there is
    // no built-in vocabulary), a missing or malformed file. Returns true.
    bool load_vocabulary(const std::string& vocab_file = "");

    std::vector<uint32_t> encode(const std::string& text, bool add_bos = true) const;
    std::string decode(const std::vector<uint32_t>& tokens, bool skip_special = true) const;
    std::string decode_single(uint32_t token, bool skip_special = true) const;

    bool is_byte_fallback(uint32_t token, uint8_t& value) const;
    bool is_special_token(uint32_t token) const;

    struct ChatMessage {
        std::string role;  // "user", "model", "system"
        std::string content;
    };
    std::string apply_chat_template(const std::vector<ChatMessage>& messages) const;

    uint32_t bos_id() const;
    uint32_t eos_id() const;
    uint32_t pad_id() const;
    uint32_t unk_id() const;
    uint32_t end_of_turn_id() const;
    uint32_t vocab_size() const;
    bool is_loaded() const;

    void set_architecture(ModelArch arch);
    ModelArch architecture() const;

    const std::vector<uint32_t>& stop_token_ids() const;

   private:
    struct Impl;
    std::unique_ptr<Impl> impl_;
    friend class IncrementalDetokenizer;
    friend class ForwardRunner;
};

}  // namespace g4dense
