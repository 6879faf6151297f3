// The container validators (csrc/format.cpp) on hand-made headers, compiled directly with the
// validator source: a well-formed header passes; a malformed one raises one error naming every
// broken rule; a wrong magic stops before the other fields are read.
#include <cstdio>
#include <cstring>
#include <string>

#include "format.h"

using namespace g4b;

static int failures = 0;
#define CHECK(c)                                                                   \
    do {                                                                           \
        if (!(c)) {                                                                \
            std::fprintf(stderr, "CHECK failed: %s (line %d)\n", #c, __LINE__);   \
            ++failures;                                                            \
        }                                                                          \
    } while (0)

static std::string error_of(const G4DenseHeader& h, uint64_t size) {
    try {
        validate_header(h, size);
    } catch (const G4DenseFormatError& e) {
        return e.what();
    }
    return "";
}

static G4DenseHeader good() {
    G4DenseHeader h;
    std::memset(&h, 0, sizeof h);
    h.magic = G4DenseHeader::kMagic;
    h.version = 3;
    h.quant_type = 1;
    h.num_layers = 2;
    h.d_model = 256;
    h.d_ff = 1024;
    h.num_q_heads = 4;
    h.num_kv_heads = 1;
    h.head_dim = 64;
    h.vocab_size = 4096;
    h.quant_group_size = 64;
    h.tied_embeddings = 1;
    h.embed_offset = h.lm_head_offset = 4096;
    // Each layer's tensors take 536 848 bytes (norms, then q, k, v, o, gate, up, down on 16-byte
    // boundaries): 140 pages hold them.
    h.layer_offsets[0] = 4096 * 200;
    h.layer_sizes[0] = 4096 * 140;
    h.layer_offsets[1] = 4096 * 340;
    h.layer_sizes[1] = 4096 * 140;
    return h;
}

int main() {
    const uint64_t size = 4096 * 480;
    CHECK(error_of(good(), size).empty());

    G4DenseHeader h = good();
    h.magic = 0x12345678;
    h.num_layers = 0;  // not reported: a foreign file stops at its magic
    std::string e = error_of(h, size);
    CHECK(e.find("magic") != std::string::npos && e.find("layers") == std::string::npos);

    h = good();
    h.layer_offsets[1] = 4096 * 340 + 8;       // unaligned (still ending inside the file)
    h.layer_sizes[1] = 4096 * 140 - 8;
    h.layer_sizes[0] = 4096 * 1000;            // past the end of the file
    h.quant_group_size = 32;                   // unsupported grouping
    e = error_of(h, size);
    CHECK(e.find("3 problems") != std::string::npos);
    CHECK(e.find("layer 1 starts at byte") != std::string::npos);
    CHECK(e.find("layer 0 ends at byte") != std::string::npos);
    CHECK(e.find("groups of 64") != std::string::npos);

    h = good();
    h.layer_offsets[0] = ~0ull - 4095;         // offset + size wraps
    CHECK(error_of(h, size).find("overflows") != std::string::npos);

    // The kernels' per-layer rules, and tensors that must fit in their layer's block.
    h = good();
    h.layer_sizes[1] = 4096 * 131;             // 536 576 bytes: 272 short
    e = error_of(h, size);
    CHECK(e.find("layer 1 holds 536576 bytes; its tensors need 536848") != std::string::npos);
    h = good();
    h.head_dim = 96;
    CHECK(error_of(h, size).find("head_dim 96") != std::string::npos);
    h = good();
    h.d_ff = 1000;
    CHECK(error_of(h, size).find("FFN width 1000") != std::string::npos);
    h = good();
    h.layer_d_ff[1] = 1040;                    // a per-layer width overrides d_ff
    CHECK(error_of(h, size).find("layer 1: FFN width 1040") != std::string::npos);
    h = good();
    h.num_q_heads = 6;
    h.num_kv_heads = 4;
    CHECK(error_of(h, size).find("whole groups") != std::string::npos);
    h = good();
    h.global_layer_mask = 0b10;                // layer 1 full-attention with head_dim 64
    h.global_head_dim = 64;
    h.global_kv_heads = 1;
    CHECK(error_of(h, size).find("too small for the 64 rotated pairs") != std::string::npos);

    G4MtpHeader m;
    std::memset(&m, 0, sizeof m);
    m.magic = G4MtpHeader::kMagic;
    m.version = 1;
    m.quant_type = 1;
    m.num_layers = 9;  // the table holds 8
    m.backbone_hidden_size = m.hidden_size = 256;
    m.intermediate_size = 512;
    m.vocab_size = 4096;
    try {
        validate_mtp_header(m, 0);
        ++failures;
    } catch (const G4DenseFormatError& x) {
        CHECK(std::string(x.what()).find("9 layers") != std::string::npos);
    }
    std::printf("{\"format_failures\": %d}\n", failures);
    return failures ? 1 : 0;
}
