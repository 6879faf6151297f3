// Text <-> token ids for Gemma-4 tokenizer.json files: the reference's Tokenizer,
// IncrementalDetokenizer and StreamingStopMatcher (include/g4dense/tokenizer.hpp:1-105,
// include/g4dense/detokenizer.hpp:1-52; src/tokenizer.cpp, src/detokenizer.cpp), with the same
// observable behaviour:
//   * encode: added tokens are taken verbatim where the text at a '<' or '[' starts one (longest
//     first); the text between them has every space replaced by U+2581 and is split by BPE --
//     start from single UTF-8 characters and repeatedly merge the adjacent pair with the lowest
//     merge rank (the leftmost of equal ranks); a final symbol that is not a vocabulary piece
//     becomes one byte-fallback token <0xNN> per byte (or <unk> without one);
//   * decode: consecutive byte-fallback tokens are fused and repaired as UTF-8 (utf8_repair);
//     other pieces have U+2581 turned back into spaces; special tokens are skipped on request;
//   * the Gemma-4 chat template (and the Muse-Glimmer one) and the stop-token set.
// BPE here keeps a heap of candidate merges over a linked list of symbols (n log n) instead of
// rescanning every pair after each merge; the merge order, and so the output, is the same.
#pragma once
#include <cstdint>
#include <string>
#include <string_view>
#include <unordered_map>
#include <vector>

namespace g4b {

// Appends the valid UTF-8 prefix of `in` to `out` (U+FFFD for a byte that cannot start a
// character) and returns the bytes consumed. An incomplete trailing sequence is held back, or
// with flush_all becomes one U+FFFD. Only lead bytes are checked: a lead byte's sequence length
// of bytes is copied as it stands.
size_t utf8_repair(std::string_view in, bool flush_all, std::string& out);

class Tokenizer {
   public:
    enum class Arch { Gemma4, MuseGlimmer };
    struct Message {
        std::string role;  // "system", "user", "model" / "assistant"
        std::string content;
    };

    // Reads a Hugging Face tokenizer.json (added_tokens, model.vocab, model.merges). Throws
    // std::runtime_error naming the problem; an empty path is an error (no built-in vocabulary).
    void load(const std::string& path);
    bool loaded() const { return loaded_; }

    std::vector<uint32_t> encode(std::string_view text, bool add_bos = true) const;
    std::string decode(const std::vector<uint32_t>& ids, bool skip_special = true) const;
    // One token's text: "" for ids outside the vocabulary and, with skip_special, special tokens;
    // otherwise its piece with U+2581 turned into spaces (byte-fallback pieces unchanged).
    std::string decode_single(uint32_t id, bool skip_special = true) const;
    bool byte_value(uint32_t id, uint8_t& value) const;  // a byte-fallback token's byte
    bool is_special(uint32_t id) const { return id < special_.size() && special_[id]; }

    // Throws std::runtime_error for a Gemma-4 system message that is not first.
    std::string chat_template(const std::vector<Message>& messages) const;

    void set_arch(Arch a);
    Arch arch() const { return arch_; }
    uint32_t bos() const { return bos_; }
    uint32_t eos() const { return eos_; }
    uint32_t pad() const { return pad_; }
    uint32_t unk() const { return unk_; }
    uint32_t end_of_turn() const { return end_of_turn_; }
    uint32_t vocab_size() const { return vocab_size_; }
    const std::vector<uint32_t>& stop_ids() const { return stop_ids_; }

   private:
    void resolve_special_ids();
    void bpe(std::string_view text, std::vector<uint32_t>& out) const;

    Arch arch_ = Arch::Gemma4;
    bool loaded_ = false;
    uint32_t bos_ = 2, eos_ = 1, pad_ = 0, unk_ = 3;
    uint32_t turn_ = 105, end_of_turn_ = 106, tool_response_ = 50;
    uint32_t vocab_size_ = 262144;
    std::vector<uint32_t> stop_ids_{1, 106, 50};
    std::vector<std::string> pieces_;                   // id -> piece
    std::unordered_map<std::string, uint32_t> ids_;     // piece -> id
    std::unordered_map<std::string, uint32_t> ranks_;   // "left\0right" -> merge rank
    std::vector<std::pair<std::string, uint32_t>> added_;  // longest first
    std::vector<bool> special_;
    int32_t byte_id_[256];
};

// Streams token ids to text that never splits a UTF-8 character: byte-fallback bytes are held
// until they complete one; any other piece first ends the byte run (repairing it).
class IncrementalDetokenizer {
   public:
    explicit IncrementalDetokenizer(const Tokenizer& t, bool skip_special = true) : t_(t), skip_(skip_special) {}
    std::string push(uint32_t id);
    std::string finish();
    void reset() { pending_.clear(); }

   private:
    std::string drain(bool flush_all);
    const Tokenizer& t_;
    bool skip_;
    std::string pending_;
};

// Stops a text stream at the earliest occurrence of any stop string, withholding a tail that
// could still become one.
class StreamingStopMatcher {
   public:
    StreamingStopMatcher() = default;
    explicit StreamingStopMatcher(std::vector<std::string> stops);
    std::string push(std::string_view text);
    std::string finish();
    bool stopped() const { return stopped_; }
    const std::string& matched() const { return matched_; }
    bool empty() const { return stops_.empty(); }

   private:
    std::vector<std::string> stops_;
    size_t longest_ = 0;
    std::string buf_;
    std::string matched_;
    bool stopped_ = false;
};

// The role/content pairs of a JSON array of {"role": ..., "content": ...} objects (other keys
// are ignored). Throws std::runtime_error on malformed JSON.
std::vector<Tokenizer::Message> parse_chat_messages(std::string_view json);

}  // namespace g4b
