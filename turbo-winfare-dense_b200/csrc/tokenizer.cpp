#include "tokenizer.h"

#include <algorithm>
#include <cstring>
#include <fstream>
#include <functional>
#include <queue>
#include <sstream>
#include <stdexcept>

namespace g4b {

namespace {

constexpr std::string_view kSpace = "\xe2\x96\x81";  // U+2581, the normalizer's stand-in for ' '

[[noreturn]] void bad(const std::string& what) { throw std::runtime_error("tokenizer.json: " + what); }

// A forward-only JSON reader: values are consumed in document order and the caller decides, key
// by key, which to read and which to skip, so a 32 MB tokenizer.json is never held as a tree.
class JsonReader {
   public:
    JsonReader(std::string_view s, const char* what) : s_(s), what_(what) {}

    void ws() {
        while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\r' || s_[i_] == '\t')) ++i_;
    }
    char peek() {
        ws();
        return i_ < s_.size() ? s_[i_] : '\0';
    }
    void eat(char c) {
        if (peek() != c) fail(std::string("expected '") + c + "' at byte " + std::to_string(i_));
        ++i_;
    }
    std::string str() {
        eat('"');
        std::string out;
        while (i_ < s_.size()) {
            const char c = s_[i_++];
            if (c == '"') return out;
            if (c != '\\') {
                out += c;
                continue;
            }
            if (i_ >= s_.size()) break;
            const char e = s_[i_++];
            switch (e) {
                case '"': out += '"'; break;
                case '\\': out += '\\'; break;
                case '/': out += '/'; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'n': out += '\n'; break;
                case 'r': out += '\r'; break;
                case 't': out += '\t'; break;
                case 'u': {
                    uint32_t cp = hex4();
                    // A high surrogate followed by an escaped low surrogate is one code point.
                    if (cp >= 0xD800 && cp < 0xDC00 && i_ + 6 <= s_.size() && s_[i_] == '\\' && s_[i_ + 1] == 'u') {
                        const size_t back = i_;
                        i_ += 2;
                        const uint32_t lo = hex4();
                        if (lo >= 0xDC00 && lo < 0xE000) cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                        else i_ = back;
                    }
                    put_utf8(out, cp);
                    break;
                }
                default: fail("bad escape at byte " + std::to_string(i_));
            }
        }
        fail("unterminated string");
    }
    long long integer() {
        ws();
        const size_t b = i_;
        if (i_ < s_.size() && (s_[i_] == '-' || s_[i_] == '+')) ++i_;
        while (i_ < s_.size() && s_[i_] >= '0' && s_[i_] <= '9') ++i_;
        if (b == i_ || (i_ - b == 1 && (s_[b] == '-' || s_[b] == '+'))) fail("expected an integer at byte " + std::to_string(b));
        // (a fraction or exponent would follow an integer id only in a malformed file)
        return std::stoll(std::string(s_.substr(b, i_ - b)));
    }
    bool boolean() {
        ws();
        if (s_.compare(i_, 4, "true") == 0) {
            i_ += 4;
            return true;
        }
        if (s_.compare(i_, 5, "false") == 0) {
            i_ += 5;
            return false;
        }
        skip();  // null or anything else reads as false
        return false;
    }
    void skip() {
        const char c = peek();
        if (c == '"') {
            str();
        } else if (c == '{') {
            object([&](const std::string&) { skip(); });
        } else if (c == '[') {
            array([&] { skip(); });
        } else {
            while (i_ < s_.size() && s_[i_] != ',' && s_[i_] != '}' && s_[i_] != ']' && s_[i_] != ' ' &&
                   s_[i_] != '\n' && s_[i_] != '\r' && s_[i_] != '\t')
                ++i_;
        }
    }
    // Calls f(key) for every member; f must consume the member's value.
    void object(const std::function<void(const std::string&)>& f) {
        eat('{');
        if (peek() == '}') {
            ++i_;
            return;
        }
        for (;;) {
            const std::string k = str();
            eat(':');
            f(k);
            const char c = peek();
            ++i_;
            if (c == '}') return;
            if (c != ',') fail("expected ',' or '}' at byte " + std::to_string(i_ - 1));
        }
    }
    // Calls f() for every element; f must consume it.
    void array(const std::function<void()>& f) {
        eat('[');
        if (peek() == ']') {
            ++i_;
            return;
        }
        for (;;) {
            f();
            const char c = peek();
            ++i_;
            if (c == ']') return;
            if (c != ',') fail("expected ',' or ']' at byte " + std::to_string(i_ - 1));
        }
    }

   private:
    uint32_t hex4() {
        if (i_ + 4 > s_.size()) fail("truncated \\u escape");
        uint32_t v = 0;
        for (int k = 0; k < 4; ++k) {
            const char c = s_[i_++];
            v <<= 4;
            if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
            else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
            else fail("bad hex digit in \\u escape");
        }
        return v;
    }
    static void put_utf8(std::string& out, uint32_t cp) {
        if (cp < 0x80) {
            out += (char)cp;
        } else if (cp < 0x800) {
            out += (char)(0xC0 | (cp >> 6));
            out += (char)(0x80 | (cp & 0x3F));
        } else if (cp < 0x10000) {
            out += (char)(0xE0 | (cp >> 12));
            out += (char)(0x80 | ((cp >> 6) & 0x3F));
            out += (char)(0x80 | (cp & 0x3F));
        } else {
            out += (char)(0xF0 | (cp >> 18));
            out += (char)(0x80 | ((cp >> 12) & 0x3F));
            out += (char)(0x80 | ((cp >> 6) & 0x3F));
            out += (char)(0x80 | (cp & 0x3F));
        }
    }

    [[noreturn]] void fail(const std::string& m) const { throw std::runtime_error(std::string(what_) + ": " + m); }

    std::string_view s_;
    const char* what_;
    size_t i_ = 0;
};

// Bytes of the UTF-8 character whose lead byte is `c` (1 for anything that is not a lead byte of
// a longer sequence).
size_t utf8_span(unsigned char c) {
    if ((c & 0xF8) == 0xF0) return 4;
    if ((c & 0xF0) == 0xE0) return 3;
    if ((c & 0xE0) == 0xC0) return 2;
    return 1;
}

// The byte of a "<0xNN>" piece, or -1.
int byte_piece(const std::string& p) {
    if (p.size() != 6 || p.compare(0, 3, "<0x") != 0 || p[5] != '>') return -1;
    auto hex = [](char c) {
        if (c >= '0' && c <= '9') return c - '0';
        if (c >= 'a' && c <= 'f') return c - 'a' + 10;
        if (c >= 'A' && c <= 'F') return c - 'A' + 10;
        return -1;
    };
    const int h = hex(p[3]), l = hex(p[4]);
    return h < 0 || l < 0 ? -1 : h * 16 + l;
}

std::string trim(const std::string& s) {
    const size_t b = s.find_first_not_of(" \t\r\n");
    if (b == std::string::npos) return "";
    const size_t e = s.find_last_not_of(" \t\r\n");
    return s.substr(b, e - b + 1);
}

}  // namespace

size_t utf8_repair(std::string_view in, bool flush_all, std::string& out) {
    static constexpr std::string_view kReplacement = "\xEF\xBF\xBD";  // U+FFFD
    size_t i = 0;
    while (i < in.size()) {
        const unsigned char c = (unsigned char)in[i];
        size_t need = 0;
        if (c < 0x80) need = 1;
        else if ((c & 0xE0) == 0xC0) need = 2;
        else if ((c & 0xF0) == 0xE0) need = 3;
        else if ((c & 0xF8) == 0xF0) need = 4;
        if (need == 0) {  // a continuation byte or an invalid lead: replace it, move on one byte
            out += kReplacement;
            ++i;
            continue;
        }
        if (i + need > in.size()) {  // an incomplete tail
            if (!flush_all) break;
            out += kReplacement;
            i = in.size();
            break;
        }
        out.append(in.data() + i, need);
        i += need;
    }
    return i;
}

void Tokenizer::load(const std::string& path) {
    if (path.empty()) throw std::runtime_error("Tokenizer::load: no vocabulary path (there is no built-in vocabulary)");
    std::ifstream f(path, std::ios::binary);
    if (!f) throw std::runtime_error("Failed to open tokenizer: " + path);
    std::ostringstream ss;
    ss << f.rdbuf();
    const std::string text = ss.str();
    if (text.empty()) throw std::runtime_error("Empty tokenizer file: " + path);

    pieces_.clear();
    ids_.clear();
    ranks_.clear();
    added_.clear();
    special_.clear();
    std::fill(byte_id_, byte_id_ + 256, -1);
    bool have_model = false, have_vocab = false;
    JsonReader r(text, "tokenizer.json");
    r.object([&](const std::string& key) {
        if (key == "added_tokens") {
            r.array([&] {
                long long id = 0;  // an entry without an id takes id 0
                std::string content;
                bool special = false;
                r.object([&](const std::string& k) {
                    if (k == "id") id = r.integer();
                    else if (k == "content") content = r.str();
                    else if (k == "special") special = r.boolean();
                    else r.skip();
                });
                if (content.empty()) return;
                if (id < 0 || id >= (1ll << 24)) bad("added token id out of range");
                added_.emplace_back(content, (uint32_t)id);
                if ((size_t)id >= special_.size()) special_.resize((size_t)id + 1, false);
                special_[(size_t)id] = special;
            });
        } else if (key == "model") {
            have_model = true;
            r.object([&](const std::string& k) {
                if (k == "vocab") {
                    have_vocab = true;
                    r.object([&](const std::string& piece) {
                        const long long id = r.integer();
                        if (id < 0 || id >= (1ll << 24)) bad("vocabulary id out of range");
                        if ((size_t)id >= pieces_.size()) pieces_.resize((size_t)id + 1);
                        pieces_[(size_t)id] = piece;
                        ids_[piece] = (uint32_t)id;  // a repeated piece keeps its last id
                        const int b = byte_piece(piece);
                        if (b >= 0) byte_id_[b] = (int32_t)id;
                    });
                } else if (k == "merges") {
                    uint32_t rank = 0;
                    r.array([&] {
                        std::string left, right;
                        if (r.peek() == '[') {  // ["left", "right"]
                            int n = 0;
                            r.array([&] {
                                if (n == 0) left = r.str();
                                else if (n == 1) right = r.str();
                                else r.skip();
                                ++n;
                            });
                        } else {  // "left right"
                            const std::string joined = r.str();
                            const size_t sp = joined.find(' ');
                            if (sp == std::string::npos) return;  // not a merge: takes no rank
                            left = joined.substr(0, sp);
                            right = joined.substr(sp + 1);
                        }
                        ranks_.emplace(left + '\0' + right, rank++);  // a repeated pair keeps its first rank
                    });
                } else {
                    r.skip();
                }
            });
        } else {
            r.skip();
        }
    });
    if (!have_model) bad("no \"model\" section");
    if (!have_vocab) bad("no model.vocab");
    if (pieces_.empty() || ids_.empty()) bad("vocabulary is empty");
    vocab_size_ = (uint32_t)pieces_.size();
    special_.resize(pieces_.size(), false);
    resolve_special_ids();
    // Longest first, so a longer added token wins over one that is its prefix.
    std::sort(added_.begin(), added_.end(), [](const auto& a, const auto& b) {
        return a.first.size() != b.first.size() ? a.first.size() > b.first.size() : a.first < b.first;
    });
    loaded_ = true;
}

void Tokenizer::resolve_special_ids() {
    auto find = [&](const char* name, uint32_t& id) {
        const auto it = ids_.find(name);
        if (it != ids_.end()) id = it->second;
    };
    if (arch_ == Arch::MuseGlimmer) {
        bos_ = 200000;
        eos_ = 200001;
        find("<|begin_of_text|>", bos_);
        find("<|start|>", bos_);
        find("<|end_of_text|>", eos_);
        uint32_t eot = 200008;
        find("<|eot|>", eot);
        stop_ids_ = {eos_, eot};
    } else {
        bos_ = 2;
        eos_ = 1;
        find("<bos>", bos_);
        find("<eos>", eos_);
        find("<pad>", pad_);
        find("<unk>", unk_);
        find("<|turn>", turn_);
        find("<turn|>", end_of_turn_);
        find("<|tool_response>", tool_response_);
        stop_ids_ = {eos_, end_of_turn_, tool_response_};
    }
}

void Tokenizer::set_arch(Arch a) {
    arch_ = a;
    if (pieces_.empty()) vocab_size_ = a == Arch::MuseGlimmer ? 202048u : 262144u;
    resolve_special_ids();
}

void Tokenizer::bpe(std::string_view text, std::vector<uint32_t>& out) const {
    if (text.empty()) return;
    // Symbols are contiguous slices of `text`, kept in a doubly linked list.
    struct Sym {
        uint32_t start, len;
        int prev, next;
    };
    std::vector<Sym> sy;
    for (size_t i = 0; i < text.size();) {
        const size_t n = std::min(utf8_span((unsigned char)text[i]), text.size() - i);
        sy.push_back({(uint32_t)i, (uint32_t)n, (int)sy.size() - 1, (int)sy.size() + 1});
        i += n;
    }
    sy.back().next = -1;
    // Candidate merges ordered by (rank, position of the left symbol): the lowest rank first,
    // the leftmost of equal ranks first. An entry is stale once either symbol has changed.
    struct Cand {
        uint32_t rank, start, llen, rlen;
        int left;
        bool operator>(const Cand& o) const { return rank != o.rank ? rank > o.rank : start > o.start; }
    };
    std::priority_queue<Cand, std::vector<Cand>, std::greater<Cand>> heap;
    std::string key;
    auto consider = [&](int l) {
        if (l < 0 || sy[l].next < 0) return;
        const Sym &a = sy[l], &b = sy[sy[l].next];
        key.assign(text.substr(a.start, a.len));
        key += '\0';
        key.append(text.substr(b.start, b.len));
        const auto it = ranks_.find(key);
        if (it != ranks_.end()) heap.push({it->second, a.start, a.len, b.len, l});
    };
    for (int l = 0; l < (int)sy.size(); ++l) consider(l);
    while (!heap.empty()) {
        const Cand c = heap.top();
        heap.pop();
        Sym& a = sy[c.left];
        if (a.len != c.llen || a.next < 0 || sy[a.next].len != c.rlen) continue;  // stale
        const int r = a.next;
        a.len += sy[r].len;
        a.next = sy[r].next;
        if (a.next >= 0) sy[a.next].prev = c.left;
        sy[r].len = 0;  // (unlinked)
        consider(a.prev);
        consider(c.left);
    }
    for (int l = 0; l >= 0; l = sy[l].next) {
        const std::string piece(text.substr(sy[l].start, sy[l].len));
        const auto it = ids_.find(piece);
        if (it != ids_.end()) {
            out.push_back(it->second);
            continue;
        }
        for (unsigned char b : piece) out.push_back(byte_id_[b] >= 0 ? (uint32_t)byte_id_[b] : unk_);
    }
}

std::vector<uint32_t> Tokenizer::encode(std::string_view text, bool add_bos) const {
    if (!loaded_) throw std::runtime_error("Tokenizer::encode called before a vocabulary was loaded");
    std::vector<uint32_t> out;
    if (add_bos) out.push_back(bos_);
    std::string run;  // text between added tokens, spaces already replaced
    auto flush = [&] {
        bpe(run, out);
        run.clear();
    };
    for (size_t i = 0; i < text.size();) {
        if (text[i] == '<' || text[i] == '[') {
            bool hit = false;
            for (const auto& [content, id] : added_)
                if (text.compare(i, content.size(), content) == 0) {
                    flush();
                    out.push_back(id);
                    i += content.size();
                    hit = true;
                    break;
                }
            if (hit) continue;
        }
        if (text[i] == ' ') run.append(kSpace);
        else run += text[i];
        ++i;
    }
    flush();
    return out;
}

bool Tokenizer::byte_value(uint32_t id, uint8_t& value) const {
    if (id >= pieces_.size()) return false;
    const int b = byte_piece(pieces_[id]);
    if (b < 0) return false;
    value = (uint8_t)b;
    return true;
}

std::string Tokenizer::decode_single(uint32_t id, bool skip_special) const {
    if (id >= pieces_.size() || (skip_special && is_special(id))) return "";
    const std::string& p = pieces_[id];
    std::string out;
    out.reserve(p.size());
    for (size_t i = 0; i < p.size();) {
        if (p.compare(i, kSpace.size(), kSpace) == 0) {
            out += ' ';
            i += kSpace.size();
        } else {
            out += p[i++];
        }
    }
    return out;
}

std::string Tokenizer::decode(const std::vector<uint32_t>& ids, bool skip_special) const {
    if (!loaded_) throw std::runtime_error("Tokenizer::decode called before a vocabulary was loaded");
    std::string out, bytes;
    for (uint32_t id : ids) {
        if (id >= pieces_.size()) continue;
        uint8_t b = 0;
        if (byte_value(id, b)) {
            bytes += (char)b;
            continue;
        }
        if (!bytes.empty()) {
            utf8_repair(bytes, true, out);
            bytes.clear();
        }
        out += decode_single(id, skip_special);
    }
    if (!bytes.empty()) utf8_repair(bytes, true, out);
    return out;
}

std::string Tokenizer::chat_template(const std::vector<Message>& messages) const {
    std::string out;
    if (arch_ == Arch::MuseGlimmer) {
        for (const Message& m : messages)
            out += "<|start|>" + (m.role == "model" ? std::string("assistant") : m.role) + "\n<|message|>" +
                   trim(m.content) + "<|eot|>\n";
        return out + "<|start|>assistant\n<|message|>";
    }
    out = "<bos>";
    for (size_t i = 0; i < messages.size(); ++i) {
        const Message& m = messages[i];
        if (m.role == "system" && i != 0) throw std::runtime_error("chat template: a system message must come first");
        out += "<|turn>" + (m.role == "assistant" ? std::string("model") : m.role) + "\n" + trim(m.content) +
               "<turn|>\n";
    }
    // the generation prompt, with thinking disabled
    return out + "<|turn>model\n<|channel>thought\n<channel|>";
}

std::string IncrementalDetokenizer::drain(bool flush_all) {
    std::string out;
    pending_.erase(0, utf8_repair(pending_, flush_all, out));
    return out;
}

std::string IncrementalDetokenizer::push(uint32_t id) {
    uint8_t b = 0;
    if (t_.byte_value(id, b)) {
        pending_ += (char)b;
        return drain(false);
    }
    if (skip_ && t_.is_special(id)) return drain(true);  // a special token ends any byte run
    std::string out = drain(true);
    pending_ += t_.decode_single(id, skip_);
    out += drain(false);
    return out;
}

std::string IncrementalDetokenizer::finish() { return drain(true); }

StreamingStopMatcher::StreamingStopMatcher(std::vector<std::string> stops) {
    for (auto& s : stops)
        if (!s.empty()) {  // an empty stop string would match at once
            longest_ = std::max(longest_, s.size());
            stops_.push_back(std::move(s));
        }
}

std::string StreamingStopMatcher::push(std::string_view text) {
    if (stopped_) return {};
    if (stops_.empty()) return std::string(text);
    buf_.append(text);
    size_t at = std::string::npos;
    const std::string* hit = nullptr;
    for (const std::string& s : stops_) {  // the earliest occurrence wins
        const size_t p = buf_.find(s);
        if (p != std::string::npos && p < at) {
            at = p;
            hit = &s;
        }
    }
    if (hit) {
        stopped_ = true;
        matched_ = *hit;
        std::string out = buf_.substr(0, at);
        buf_.clear();
        return out;
    }
    // Withhold the longest tail (shorter than the longest stop) that begins some stop string.
    size_t hold = 0;
    for (size_t n = std::min(longest_ ? longest_ - 1 : 0, buf_.size()); n >= 1 && !hold; --n)
        for (const std::string& s : stops_)
            if (s.size() > n && s.compare(0, n, buf_, buf_.size() - n, n) == 0) {
                hold = n;
                break;
            }
    std::string out = buf_.substr(0, buf_.size() - hold);
    buf_.erase(0, buf_.size() - hold);
    return out;
}

std::string StreamingStopMatcher::finish() {
    if (stopped_) return {};
    std::string out;
    out.swap(buf_);
    return out;
}

std::vector<Tokenizer::Message> parse_chat_messages(std::string_view json) {
    std::vector<Tokenizer::Message> out;
    JsonReader r(json, "chat messages JSON");
    r.array([&] {
        Tokenizer::Message m;
        r.object([&](const std::string& k) {
            if (k == "role") m.role = r.str();
            else if (k == "content") m.content = r.str();
            else r.skip();
        });
        out.push_back(std::move(m));
    });
    return out;
}

}  // namespace g4b
