// The public C++ tokenizer API (include/g4dense/tokenizer.hpp, detokenizer.hpp) and
// ForwardRunner::generate's text path, exercised the way the reference's own C++ tests use them
// (tests/test_tokenizer.cpp, tests/test_detokenizer.cpp of the reference).
//
//   test_tokenizer_api cpu <dir for scratch files>
//   test_tokenizer_api gpu <container> <tokenizer.json> <prompt> <max_tokens>
//       prints one JSON line {"tokens": [...], "pieces": ["hex", ...]} from ForwardRunner::generate
//       (greedy, chat template on).
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <random>
#include <string>
#include <vector>

#include "g4dense/detokenizer.hpp"
#include "g4dense/runner.hpp"
#include "g4dense/tokenizer.hpp"

using namespace g4dense;

static int g_fail = 0;
#define CHECK(c)                                                             \
    do {                                                                     \
        if (!(c)) {                                                          \
            std::printf("FAIL %s:%d: %s\n", __FILE__, __LINE__, #c);        \
            ++g_fail;                                                        \
        }                                                                    \
    } while (0)

template <class F>
static bool throws_format_error(F&& f) {
    try {
        f();
    } catch (const G4DenseFormatError&) {
        return true;
    } catch (...) {
        return false;
    }
    return false;
}

static std::string write(const std::string& path, const std::string& text) {
    std::ofstream(path, std::ios::binary | std::ios::trunc) << text;
    return path;
}

static int cpu(const std::string& dir) {
    // Default state: no vocabulary, Gemma-4 special ids and stop set {1, 106, 50}.
    Tokenizer tok;
    CHECK(!tok.is_loaded());
    CHECK(tok.vocab_size() == 262144 && tok.bos_id() == 2 && tok.eos_id() == 1 && tok.pad_id() == 0);
    CHECK(tok.unk_id() == 3 && tok.end_of_turn_id() == 106);
    CHECK((tok.stop_token_ids() == std::vector<uint32_t>{1, 106, 50}));
    CHECK(throws_format_error([&] { tok.encode("Hello", true); }));
    CHECK(throws_format_error([&] { Tokenizer t; t.load_vocabulary("definitely_not_a_real_vocab_file.json"); }));
    CHECK(throws_format_error([&] { Tokenizer t; t.load_vocabulary(); }));

    // The chat template over a mini vocabulary.
    const std::string mini = write(dir + "/mini.json",
        R"({"added_tokens": [{"id": 0, "content": "<pad>", "special": true},
             {"id": 1, "content": "<eos>", "special": true}, {"id": 2, "content": "<bos>", "special": true},
             {"id": 105, "content": "<start_of_turn>", "special": true},
             {"id": 106, "content": "<end_of_turn>", "special": true}, {"id": 107, "content": "\n", "special": false}],
            "model": {"vocab": {"<pad>": 0, "<eos>": 1, "<bos>": 2, "<start_of_turn>": 105, "<end_of_turn>": 106,
                                "\n": 107, "user": 2364, "model": 4368, "Hi": 10979}, "merges": []}})");
    Tokenizer m;
    CHECK(m.load_vocabulary(mini) && m.is_loaded());
    CHECK(m.apply_chat_template({{"user", "Hi"}}) ==
          "<bos><|turn>user\nHi<turn|>\n<|turn>model\n<|channel>thought\n<channel|>");
    CHECK(throws_format_error([&] { m.apply_chat_template({{"user", "a"}, {"system", "b"}}); }));

    // Muse-Glimmer ids and template on a default-constructed tokenizer.
    Tokenizer muse;
    muse.set_architecture(ModelArch::MUSE_GLIMMER);
    CHECK(muse.architecture() == ModelArch::MUSE_GLIMMER);
    CHECK(muse.bos_id() == 200000 && muse.eos_id() == 200001 && muse.vocab_size() == 202048);
    CHECK((muse.stop_token_ids() == std::vector<uint32_t>{200001, 200008}));
    CHECK(muse.apply_chat_template({{"user", "Hello world"}}) ==
          "<|start|>user\n<|message|>Hello world<|eot|>\n<|start|>assistant\n<|message|>");

    // Detokenizer over Hi 2, " there" 3, ! 4, <0xNN> at 100 + NN.
    std::string v = R"({"added_tokens":[{"id":0,"content":"<pad>","special":true},{"id":1,"content":"<eos>","special":true}],)"
                    R"("model":{"vocab":{"<pad>":0,"<eos>":1,"Hi":2," there":3,"!":4)";
    for (int b = 0; b < 256; ++b) {
        char piece[32];
        std::snprintf(piece, sizeof(piece), ",\"<0x%02X>\":%d", b, 100 + b);
        v += piece;
    }
    v += R"(},"merges":[]}})";
    Tokenizer dt;
    dt.load_vocabulary(write(dir + "/detok.json", v));
    {
        IncrementalDetokenizer d(dt);
        CHECK(d.push(100 + 0xE2).empty() && d.push(100 + 0x82).empty());
        CHECK(d.push(100 + 0xAC) == "\xE2\x82\xAC" && d.finish().empty());
    }
    {
        IncrementalDetokenizer d(dt);
        CHECK(d.push(100 + 0xE2).empty() && d.finish() == "\xEF\xBF\xBD");
    }
    {
        IncrementalDetokenizer d(dt);
        std::string out = d.push(2);
        out += d.push(1);
        out += d.push(4);
        out += d.finish();
        CHECK(out == "Hi!");
    }
    std::mt19937_64 rng(0xD370C0D3ULL);
    for (int trial = 0; trial < 200; ++trial) {
        std::vector<uint32_t> ids(1 + rng() % 64);
        for (auto& t : ids) t = 100 + (uint32_t)(rng() % 256);
        IncrementalDetokenizer d(dt);
        std::string s;
        for (uint32_t t : ids) s += d.push(t);
        s += d.finish();
        CHECK(s == dt.decode(ids, false));
    }
    std::string repaired;
    CHECK(utf8_repair("a\xE2\x82", false, repaired) == 1 && repaired == "a");

    // Stop matcher.
    {
        StreamingStopMatcher s({"<eos>"});
        CHECK(s.push("<eos>").empty() && s.stopped() && s.matched() == "<eos>");
        StreamingStopMatcher s2({"<start_of_turn>model"});
        std::string out = s2.push("<start_of_turn>");
        CHECK(out.empty() && !s2.stopped());
        StreamingStopMatcher copy = s2;  // copies carry the withheld text
        out += s2.push("user");
        out += s2.finish();
        CHECK(!s2.stopped() && out == "<start_of_turn>user");
        CHECK(copy.push("model").empty() && copy.stopped());
        CHECK(StreamingStopMatcher().empty() && StreamingStopMatcher({""}).empty());
    }
    std::printf("%s (%d failures)\n", g_fail ? "FAILED" : "ok", g_fail);
    return g_fail ? 1 : 0;
}

static int gpu(const std::string& container, const std::string& tokp, const std::string& prompt, int n) {
    auto ctx = DeviceContext::create(0);
    auto tok = std::make_shared<Tokenizer>();
    tok->load_vocabulary(tokp);
    ForwardRunner r(ctx, tok, container);
    r.initialize();
    GenerationOptions o;
    o.max_tokens = n;
    std::vector<uint32_t> toks;
    std::vector<std::string> pieces;
    r.generate(prompt, o, [&](uint32_t t, const std::string& p) {
        toks.push_back(t);
        pieces.push_back(p);
        return true;
    });
    std::printf("{\"tokens\": [");
    for (size_t i = 0; i < toks.size(); ++i) std::printf("%s%u", i ? ", " : "", toks[i]);
    std::printf("], \"pieces\": [");
    for (size_t i = 0; i < pieces.size(); ++i) {
        std::printf("%s\"", i ? ", " : "");
        for (unsigned char c : pieces[i]) std::printf("%02x", c);
        std::printf("\"");
    }
    std::printf("]}\n");
    // Without a tokenizer the text entry point throws, as the reference's runner does.
    ForwardRunner bare(ctx, container);
    bare.initialize();
    try {
        bare.generate(prompt, o, nullptr);
        return 1;
    } catch (const std::runtime_error& e) {
        if (std::string(e.what()).find("Tokenizer is not loaded") == std::string::npos) return 1;
    }
    return 0;
}

int main(int argc, char** argv) {
    if (argc >= 3 && std::string(argv[1]) == "cpu") return cpu(argv[2]);
    if (argc >= 6 && std::string(argv[1]) == "gpu") return gpu(argv[2], argv[3], argv[4], std::atoi(argv[5]));
    std::fprintf(stderr, "usage: test_tokenizer_api cpu <dir> | gpu <container> <tokenizer.json> <prompt> <n>\n");
    return 2;
}
