// The .g4dense v3 container contract (the on-disk format is the reference's, unchanged):
// G4DenseHeader layout of include/g4dense/format.hpp:26-110, validation of
// src/format.cpp:6-65, geometry resolution of include/g4dense/format.hpp:189-241.
#pragma once
#include <cstdint>
#include <stdexcept>
#include <string>

namespace g4b {

class G4DenseFormatError : public std::runtime_error {
   public:
    explicit G4DenseFormatError(const std::string& m) : std::runtime_error(m) {}
};

#pragma pack(push, 1)
struct G4DenseHeader {
    static constexpr uint32_t kMagic = 0x4734444E;  // 'G4DN'
    static constexpr uint32_t kVersion = 3;
    static constexpr uint64_t kAlign = 4096;
    static constexpr uint32_t kMaxLayers = 60;

    uint32_t magic, version, quant_type, num_layers, d_model, d_ff, num_q_heads, num_kv_heads, head_dim,
        vocab_size, sliding_window, quant_group_size, scale_dtype, tied_embeddings;
    uint64_t global_layer_mask;
    float rope_theta_local, rope_theta_global, rope_scaling, final_logit_softcapping;
    uint64_t embed_offset, embed_size, lm_head_offset, lm_head_size;
    uint64_t layer_offsets[60];
    uint64_t layer_sizes[60];
    uint8_t payload_sha256[32];
    uint32_t global_head_dim, global_kv_heads;
    uint32_t ple_dim, ple_vocab, num_kv_shared_layers, ple_reserved;
    uint64_t ple_offset, ple_size;
    uint32_t layer_d_ff[60];
    uint32_t arch_type, attn_out_dim;
    float qk_scale_factor, output_multiplier;
    uint8_t reserved[2696];
};
#pragma pack(pop)
static_assert(sizeof(G4DenseHeader) == 4096, "G4DenseHeader must be 4096 bytes");

struct LayerGeometry {
    uint32_t head_dim, q_heads, kv_heads;
    bool is_global;
};

inline LayerGeometry resolve_layer_geometry(const G4DenseHeader& h, uint32_t l) {
    LayerGeometry g{h.head_dim, h.num_q_heads, h.num_kv_heads, ((h.global_layer_mask >> l) & 1ull) != 0};
    if (g.is_global) {
        g.head_dim = h.global_head_dim ? h.global_head_dim : 512u;
        g.kv_heads = h.global_kv_heads ? h.global_kv_heads : 4u;
    }
    return g;
}

inline uint32_t layer_ffn_width(const G4DenseHeader& h, uint32_t l) {
    return (l < G4DenseHeader::kMaxLayers && h.layer_d_ff[l] != 0) ? h.layer_d_ff[l] : h.d_ff;
}

// Throws one G4DenseFormatError naming every rule the header breaks: the format's own rules
// (magic, version, layer count, geometry, aligned blocks inside the file; the reference checks the
// same, src/format.cpp:6-65) and what this engine needs (Gemma-4 architecture, INT4 G64, no PLE,
// tied embedding).
void validate_header(const G4DenseHeader& h, uint64_t file_size);

// The .g4mtp v1 container of the MTP "assistant" drafter: G4MtpHeader of
// include/g4dense/format.hpp:143-180 (packed, 4096 bytes).
#pragma pack(push, 1)
struct G4MtpHeader {
    static constexpr uint32_t kMagic = 0x47344D54;  // 'G4MT'
    static constexpr uint32_t kVersion = 1;
    static constexpr uint64_t kAlign = 4096;
    static constexpr uint32_t kMaxLayers = 8;

    uint32_t magic, version, quant_type, num_layers, backbone_hidden_size, hidden_size, intermediate_size,
        vocab_size, num_q_heads, num_kv_heads, head_dim, global_head_dim, global_kv_heads, sliding_window;
    uint64_t global_layer_mask;
    uint32_t quant_group_size, scale_dtype;
    uint64_t embed_offset, embed_size, pre_proj_offset, pre_proj_size, post_proj_offset, post_proj_size,
        norm_offset, norm_size;
    uint64_t layer_offsets[8];
    uint64_t layer_sizes[8];
    uint8_t payload_sha256[32];
    uint8_t reserved[3800];
};
#pragma pack(pop)
static_assert(sizeof(G4MtpHeader) == 4096, "G4MtpHeader must be 4096 bytes");

// The same for the MTP drafter's header (the reference's checks: src/format.cpp:67-130).
void validate_mtp_header(const G4MtpHeader& h, uint64_t file_size);

}  // namespace g4b
