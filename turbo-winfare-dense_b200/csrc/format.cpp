// Container validation for the .g4dense v3 and .g4mtp v1 formats.
//
// The rules are the ones the formats impose (the reference enforces the same ones in
// src/format.cpp:6-130): the magic and version, a layer count inside the header's tables, non-zero
// geometry, 4096-byte aligned blocks that lie inside the file. On top of those come the rules this
// engine needs to run a model (Gemma-4 architecture, INT4 G64 weights, tied embedding, widths in
// whole 64-groups).
//
// The checks run to completion and every broken rule is reported in one G4DenseFormatError, so a
// malformed file is diagnosed in one pass instead of one rule at a time.
#include "format.h"

#include <cinttypes>
#include <cstdarg>
#include <cstdio>
#include <string>
#include <vector>

namespace g4b {

namespace {

std::string fmt(const char* f, ...) __attribute__((format(printf, 1, 2)));
std::string fmt(const char* f, ...) {
    char buf[256];
    va_list ap;
    va_start(ap, f);
    std::vsnprintf(buf, sizeof buf, f, ap);
    va_end(ap);
    return buf;
}

// Collects the rules a header breaks and raises them together.
class Findings {
   public:
    explicit Findings(const char* what) : what_(what) {}
    void expect(bool ok, std::string problem) {
        if (!ok) problems_.push_back(std::move(problem));
    }
    bool clean() const { return problems_.empty(); }
    void raise() const {
        if (problems_.empty()) return;
        std::string msg = what_;
        msg += problems_.size() == 1 ? " is malformed: " : " is malformed (" + std::to_string(problems_.size()) + " problems): ";
        for (size_t i = 0; i < problems_.size(); ++i) msg += (i ? "; " : "") + problems_[i];
        throw G4DenseFormatError(msg);
    }

   private:
    const char* what_;
    std::vector<std::string> problems_;
};

// A block of the file: starts on a 4096-byte page, has a size, and (when the file size is known)
// ends inside the file without the end overflowing 64 bits.
void check_block(Findings& f, const std::string& name, uint64_t offset, uint64_t size, uint64_t file_size,
                 uint64_t page, bool size_required) {
    f.expect(offset % page == 0, fmt("%s starts at byte %" PRIu64 ", not on a %" PRIu64 "-byte page", name.c_str(),
                                     offset, page));
    if (size_required) f.expect(size != 0, name + " is empty");
    const bool wraps = offset + size < offset;
    f.expect(!wraps, name + ": offset + size overflows 64 bits");
    if (file_size > 0 && !wraps)
        f.expect(offset + size <= file_size, fmt("%s ends at byte %" PRIu64 ", past the end of the %" PRIu64 "-byte file",
                                                 name.c_str(), offset + size, file_size));
}

// Bytes a layer's tensors take inside its block, in the layout the loader parses
// (src/cpu_reference.cpp:324-395): the bf16 norms (four [d], q_norm and k_norm [head_dim]) and the
// layer scalar, then q, k, v (absent on full-attention layers), o, gate, up and down, each starting
// on a 16-byte boundary of the block with its packed nibbles, bf16 scales and bf16 biases.
uint64_t layer_payload_bytes(const G4DenseHeader& h, uint32_t l) {
    const LayerGeometry g = resolve_layer_geometry(h, l);
    const uint64_t d = h.d_model, F = layer_ffn_width(h, l), hd = g.head_dim;
    uint64_t n = (4 * d + 2 * hd + 1) * 2;
    auto matrix = [&n](uint64_t rows, uint64_t cols) {
        n = (n + 15) / 16 * 16;
        n += rows * (cols / 8) * 4 + 2 * rows * (cols / 64) * 2;
    };
    matrix((uint64_t)g.q_heads * hd, d);
    matrix((uint64_t)g.kv_heads * hd, d);
    if (!g.is_global) matrix((uint64_t)g.kv_heads * hd, d);
    matrix(d, (uint64_t)g.q_heads * hd);
    matrix(F, d);
    matrix(F, d);
    matrix(d, F);
    return n;
}

// The per-layer rules of the kernels: attention is built for head dims 64, 128, 256 and 512, a
// full-attention layer rotates 64 pairs, query heads come in whole GQA groups, and every GEMM's
// reduction runs over whole 64-wide groups. Then the layer's tensors must fit in its block.
void check_layers(Findings& f, const G4DenseHeader& h, uint64_t file_size) {
    for (uint32_t l = 0; l < h.num_layers; ++l) {
        const LayerGeometry g = resolve_layer_geometry(h, l);
        const uint32_t F = layer_ffn_width(h, l), hd = g.head_dim;
        const std::string name = std::string(g.is_global ? "full-attention " : "sliding ") + "layer " + std::to_string(l);
        bool ok = true;
        auto rule = [&](bool c, const std::string& problem) {
            f.expect(c, name + ": " + problem);
            ok = ok && c;
        };
        rule(hd == 64 || hd == 128 || hd == 256 || hd == 512, fmt("head_dim %u; the kernels take 64, 128, 256 or 512", hd));
        rule(!g.is_global || hd >= 128, fmt("head_dim %u is too small for the 64 rotated pairs", hd));
        rule(g.kv_heads > 0 && g.q_heads > 0 && g.q_heads % g.kv_heads == 0,
             fmt("%u query heads do not form whole groups over %u KV heads", g.q_heads, g.kv_heads));
        rule(F > 0 && F % 64 == 0, fmt("FFN width %u is not a whole number of 64-wide groups", F));
        if (!ok || file_size == 0) continue;  // the size below is only meaningful for a sound geometry
        const uint64_t need = layer_payload_bytes(h, l);
        f.expect(need <= h.layer_sizes[l], fmt("%s holds %" PRIu64 " bytes; its tensors need %" PRIu64, name.c_str(),
                                               h.layer_sizes[l], need));
    }
}

}  // namespace

void validate_header(const G4DenseHeader& h, uint64_t file_size) {
    using H = G4DenseHeader;
    Findings f("g4dense container");
    f.expect(h.magic == H::kMagic, fmt("magic word is 0x%08X; a .g4dense file starts with 0x%08X ('G4DN')", h.magic,
                                       H::kMagic));
    f.expect(h.version == H::kVersion, fmt("format version %u; this library reads version %u", h.version, H::kVersion));
    if (!f.clean()) f.raise();  // not this format: the remaining fields mean nothing
    const bool layers_ok = h.num_layers >= 1 && h.num_layers <= H::kMaxLayers;
    f.expect(layers_ok, fmt("%u layers; the header's tables hold 1..%u", h.num_layers, H::kMaxLayers));
    f.expect(h.d_model && h.d_ff && h.vocab_size,
             fmt("zero-sized geometry (d_model %u, d_ff %u, vocab %u)", h.d_model, h.d_ff, h.vocab_size));
    check_block(f, "embedding block", h.embed_offset, 0, 0, H::kAlign, false);
    check_block(f, "LM head block", h.lm_head_offset, 0, 0, H::kAlign, false);
    if (layers_ok)
        for (uint32_t i = 0; i < h.num_layers; ++i)
            check_block(f, "layer " + std::to_string(i), h.layer_offsets[i], h.layer_sizes[i], file_size, H::kAlign, true);

    // What this engine runs.
    f.expect(h.quant_type == 1 && h.quant_group_size == 64,
             fmt("quantization %u with group %u; only affine INT4 in groups of 64 (type 1) is supported", h.quant_type,
                 h.quant_group_size));
    f.expect(h.arch_type == 0, fmt("architecture %u; only Gemma 4 (0) is supported", h.arch_type));
    f.expect(h.ple_dim == 0 && h.num_kv_shared_layers == 0, "per-layer embeddings and shared KV layers are not supported");
    f.expect(h.tied_embeddings == 1 && h.lm_head_offset == h.embed_offset,
             "the LM head must be the tied embedding table (same block)");
    f.expect(h.d_model % 64 == 0, fmt("d_model %u is not a whole number of 64-wide groups", h.d_model));
    // The layer rules assume the layout this engine reads (Gemma 4, no per-layer inputs).
    if (layers_ok && h.arch_type == 0 && h.ple_dim == 0 && h.num_kv_shared_layers == 0 && h.d_model % 64 == 0)
        check_layers(f, h, file_size);
    if (file_size > 0 && h.d_model % 64 == 0) {
        // Packed nibbles, bf16 scales and biases of the tied table, then the bf16 final norm.
        const uint64_t table = (uint64_t)h.vocab_size * h.d_model / 2 + (uint64_t)h.vocab_size * (h.d_model / 64) * 4 +
                               (uint64_t)h.d_model * 2;
        check_block(f, "embedding table", h.embed_offset, table, file_size, H::kAlign, false);
    }
    f.raise();
}

void validate_mtp_header(const G4MtpHeader& h, uint64_t file_size) {
    using H = G4MtpHeader;
    Findings f("g4mtp drafter container");
    f.expect(h.magic == H::kMagic, fmt("magic word is 0x%08X; a .g4mtp file starts with 0x%08X ('G4MT')", h.magic,
                                       H::kMagic));
    f.expect(h.version == H::kVersion, fmt("format version %u; this library reads version %u", h.version, H::kVersion));
    if (!f.clean()) f.raise();
    const bool layers_ok = h.num_layers >= 1 && h.num_layers <= H::kMaxLayers;
    f.expect(layers_ok, fmt("%u layers; the header's tables hold 1..%u", h.num_layers, H::kMaxLayers));
    f.expect(h.backbone_hidden_size && h.hidden_size && h.intermediate_size && h.vocab_size,
             fmt("zero-sized geometry (backbone %u, hidden %u, intermediate %u, vocab %u)", h.backbone_hidden_size,
                 h.hidden_size, h.intermediate_size, h.vocab_size));
    struct Section {
        const char* name;
        uint64_t offset;
    };
    for (const Section& s : {Section{"embedding section", h.embed_offset}, Section{"pre-projection section", h.pre_proj_offset},
                             Section{"post-projection section", h.post_proj_offset}, Section{"norm section", h.norm_offset}})
        check_block(f, s.name, s.offset, 0, 0, H::kAlign, false);
    if (layers_ok)
        for (uint32_t i = 0; i < h.num_layers; ++i)
            check_block(f, "drafter layer " + std::to_string(i), h.layer_offsets[i], h.layer_sizes[i], file_size,
                        H::kAlign, true);

    // What this engine runs.
    f.expect(h.quant_type == 1 && (h.quant_group_size == 0 || h.quant_group_size == 64),
             fmt("quantization %u with group %u; only affine INT4 in groups of 64 is supported", h.quant_type,
                 h.quant_group_size));
    f.expect(h.hidden_size % 64 == 0 && h.intermediate_size % 64 == 0 && h.backbone_hidden_size % 64 == 0,
             "hidden, intermediate and backbone widths must be whole numbers of 64-wide groups");
    f.raise();
}

}  // namespace g4b
