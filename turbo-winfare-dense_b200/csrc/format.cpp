#include "format.h"

#include <sstream>
#include <utility>

namespace g4b {

void validate_header(const G4DenseHeader& h, uint64_t file_size) {
    if (h.magic != G4DenseHeader::kMagic) {
        std::stringstream ss;
        ss << "Invalid magic: expected 0x" << std::hex << G4DenseHeader::kMagic << ", got 0x" << h.magic;
        throw G4DenseFormatError(ss.str());
    }
    if (h.version != G4DenseHeader::kVersion) {
        std::stringstream ss;
        ss << "Unsupported container version: expected " << G4DenseHeader::kVersion << ", got " << h.version;
        throw G4DenseFormatError(ss.str());
    }
    if (h.num_layers == 0 || h.num_layers > G4DenseHeader::kMaxLayers) {
        std::stringstream ss;
        ss << "Invalid layer count: " << h.num_layers << " (max " << G4DenseHeader::kMaxLayers << ")";
        throw G4DenseFormatError(ss.str());
    }
    if (h.d_model == 0 || h.d_ff == 0 || h.vocab_size == 0)
        throw G4DenseFormatError("Invalid model geometry dimensions (d_model, d_ff, or vocab_size is zero)");
    if (h.embed_offset % G4DenseHeader::kAlign != 0) throw G4DenseFormatError("Embedding offset is not 4096-byte aligned");
    if (h.lm_head_offset % G4DenseHeader::kAlign != 0) throw G4DenseFormatError("LM head offset is not 4096-byte aligned");
    for (uint32_t i = 0; i < h.num_layers; ++i) {
        if (h.layer_offsets[i] % G4DenseHeader::kAlign != 0) {
            std::stringstream ss;
            ss << "Layer " << i << " offset (" << h.layer_offsets[i] << ") is not 4096-byte aligned";
            throw G4DenseFormatError(ss.str());
        }
        if (h.layer_sizes[i] == 0) {
            std::stringstream ss;
            ss << "Layer " << i << " has size 0";
            throw G4DenseFormatError(ss.str());
        }
        if (h.layer_offsets[i] + h.layer_sizes[i] < h.layer_offsets[i]) throw G4DenseFormatError("layer bounds: arithmetic overflow");
        if (file_size > 0 && h.layer_offsets[i] + h.layer_sizes[i] > file_size) {
            std::stringstream ss;
            ss << "Layer " << i << " extends beyond file bounds (offset=" << h.layer_offsets[i]
               << ", size=" << h.layer_sizes[i] << ", file_size=" << file_size << ")";
            throw G4DenseFormatError(ss.str());
        }
    }
    // What this engine implements.
    if (h.quant_type != 1 || h.quant_group_size != 64)
        throw G4DenseFormatError("Unsupported quantization: only AFFINE_INT4_G64 is implemented");
    if (h.arch_type != 0) throw G4DenseFormatError("Unsupported architecture: only Gemma 4 is implemented");
    if (h.ple_dim != 0 || h.num_kv_shared_layers != 0)
        throw G4DenseFormatError("Per-layer embeddings / KV sharing are not implemented");
    if (h.tied_embeddings != 1 || h.lm_head_offset != h.embed_offset)
        throw G4DenseFormatError("Only tied embedding / LM head containers are supported");
    if (h.d_model % 64 || h.vocab_size == 0) throw G4DenseFormatError("d_model must be a multiple of 64");
    if (file_size > 0) {
        const uint64_t emb = (uint64_t)h.vocab_size * (h.d_model / 8) * 4 + (uint64_t)h.vocab_size * (h.d_model / 64) * 4 +
                             (uint64_t)h.d_model * 2;
        if (h.embed_offset + emb > file_size) throw G4DenseFormatError("Embedding block extends beyond file bounds");
    }
}

void validate_mtp_header(const G4MtpHeader& h, uint64_t file_size) {
    if (h.magic != G4MtpHeader::kMagic) {
        std::stringstream ss;
        ss << "Invalid MTP magic: expected 0x" << std::hex << G4MtpHeader::kMagic << ", got 0x" << h.magic;
        throw G4DenseFormatError(ss.str());
    }
    if (h.version != G4MtpHeader::kVersion) {
        std::stringstream ss;
        ss << "Unsupported MTP container version: expected " << G4MtpHeader::kVersion << ", got " << h.version;
        throw G4DenseFormatError(ss.str());
    }
    if (h.num_layers == 0 || h.num_layers > G4MtpHeader::kMaxLayers) {
        std::stringstream ss;
        ss << "Invalid MTP layer count: " << h.num_layers << " (max " << G4MtpHeader::kMaxLayers << ")";
        throw G4DenseFormatError(ss.str());
    }
    if (h.backbone_hidden_size == 0 || h.hidden_size == 0 || h.intermediate_size == 0 || h.vocab_size == 0)
        throw G4DenseFormatError(
            "Invalid MTP model geometry dimensions (backbone_hidden, hidden_size, or vocab_size is zero)");
    const std::pair<uint64_t, const char*> aligned[] = {{h.embed_offset, "embedding"},
                                                        {h.pre_proj_offset, "pre-projection"},
                                                        {h.post_proj_offset, "post-projection"},
                                                        {h.norm_offset, "norm"}};
    for (const auto& a : aligned)
        if (a.first % G4MtpHeader::kAlign != 0)
            throw G4DenseFormatError(std::string("MTP ") + a.second + " offset is not 4096-byte aligned");
    for (uint32_t i = 0; i < h.num_layers; ++i) {
        if (h.layer_offsets[i] % G4MtpHeader::kAlign != 0) {
            std::stringstream ss;
            ss << "MTP Layer " << i << " offset (" << h.layer_offsets[i] << ") is not 4096-byte aligned";
            throw G4DenseFormatError(ss.str());
        }
        if (h.layer_sizes[i] == 0) {
            std::stringstream ss;
            ss << "MTP Layer " << i << " has size 0";
            throw G4DenseFormatError(ss.str());
        }
        if (h.layer_offsets[i] + h.layer_sizes[i] < h.layer_offsets[i])
            throw G4DenseFormatError("Integer overflow in MTP layer bounds");
        if (file_size > 0 && h.layer_offsets[i] + h.layer_sizes[i] > file_size) {
            std::stringstream ss;
            ss << "MTP Layer " << i << " extends beyond file bounds (offset=" << h.layer_offsets[i]
               << ", size=" << h.layer_sizes[i] << ", file_size=" << file_size << ")";
            throw G4DenseFormatError(ss.str());
        }
    }
    // Beyond the reference's checks: what this engine needs to run the drafter.
    if (h.quant_type != 1 || (h.quant_group_size != 0 && h.quant_group_size != 64))
        throw G4DenseFormatError("MTP container: only INT4 G64 weights are supported");
    if (h.hidden_size % 64 || h.intermediate_size % 64 || h.backbone_hidden_size % 64)
        throw G4DenseFormatError("MTP container: widths must be multiples of 64");
}

}  // namespace g4b
