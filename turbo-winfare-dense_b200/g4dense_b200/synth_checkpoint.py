"""Synthetic MLX-style checkpoints (config.json + *.safetensors) for the converter's tests; no real
checkpoint is available here.

`gemma4_tensors(spec, seed)` draws the tensors of a Gemma-4 dense model in exactly the order and
with the distributions of `container.build_container(spec, seed)`: converting the checkpoint
must reproduce that container's payload. Quantized matrices are MLX affine INT4 group-64:
`<name>.weight` packed uint32 `[rows][cols/8]`, `<name>.scales` and `<name>.biases` bf16
`[rows][cols/64]`. Full-attention layers carry no v_proj (their V is the raw K), as in the
container. `assistant_tensors(spec, seed)` does the same for an MTP assistant drafter and
`container.build_mtp_container`. `converter_cases()` and `assistant_cases()` are the checkpoints
the converters are pinned on against the reference's converters. `e2b_tensors` draws an
E2B-style model (per-layer inputs, shared-KV layers), and `forward_cases()` lists the
checkpoints on which the reference's NumPy forward pass pins converter and oracle.
`write_checkpoint` lays any tensor dict out as safetensors shards under a name prefix.
"""
from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np

from .container import ModelSpec, MtpSpec, _norm, f32_to_bf16_bits, random_quant_block

PROJ_NAMES = {"q": "self_attn.q_proj", "k": "self_attn.k_proj", "v": "self_attn.v_proj", "o": "self_attn.o_proj",
              "gate": "mlp.gate_proj", "up": "mlp.up_proj", "down": "mlp.down_proj"}


def _bf16(bits: np.ndarray):
    return ("BF16", list(bits.shape), bits.tobytes())


def quant_tensors(name: str, packed, scales, biases) -> dict:
    return {name + ".weight": ("U32", list(packed.shape), packed.tobytes()),
            name + ".scales": _bf16(scales), name + ".biases": _bf16(biases)}


def gemma4_tensors(spec: ModelSpec, seed: int = 0, centered: bool = False) -> dict:
    """name -> (safetensors dtype, shape, raw bytes), drawn as container.build_container draws."""
    rng = np.random.default_rng(seed)
    d = spec.d_model
    out = quant_tensors("embed_tokens", *random_quant_block(rng, spec.vocab_size, d, centered))
    out["norm.weight"] = _bf16(_norm(rng, d))
    scalar = f32_to_bf16_bits(np.array([1.0 / np.sqrt(2.0 * spec.num_layers)], dtype=np.float32))
    for l in range(spec.num_layers):
        hd = spec.layer_geometry(l)[0]
        pre = f"layers.{l}."
        for n in ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
                  "post_feedforward_layernorm"):
            out[pre + n + ".weight"] = _bf16(_norm(rng, d))
        out[pre + "self_attn.q_norm.weight"] = _bf16(_norm(rng, hd))
        out[pre + "self_attn.k_norm.weight"] = _bf16(_norm(rng, hd))
        out[pre + "layer_scalar"] = _bf16(scalar)
        for short, rows, cols in spec.layer_projections(l):
            out.update(quant_tensors(pre + PROJ_NAMES[short], *random_quant_block(rng, rows, cols, centered)))
    return out


def gemma4_config(spec: ModelSpec) -> dict:
    """config.json for `spec` in the Hugging Face Gemma-4 layout (fields under text_config),
    stating every value the container header records so none falls back to a default."""
    gmask = spec.global_layer_mask
    return {
        "architectures": ["Gemma4ForConditionalGeneration"],
        "model_type": "gemma4",
        "text_config": {
            "num_hidden_layers": spec.num_layers, "hidden_size": spec.d_model, "intermediate_size": spec.d_ff,
            "num_attention_heads": spec.num_q_heads, "num_key_value_heads": spec.num_kv_heads,
            "head_dim": spec.head_dim, "vocab_size": spec.vocab_size, "sliding_window": spec.sliding_window,
            "global_head_dim": spec.global_head_dim or (spec.head_dim if gmask == 0 else 512),
            "num_global_key_value_heads": spec.global_kv_heads or (spec.num_kv_heads if gmask == 0 else 4),
            "final_logit_softcapping": spec.softcap, "tie_word_embeddings": True,
            "rope_parameters": {"sliding_attention": {"rope_theta": spec.rope_theta_local},
                                "full_attention": {"rope_theta": spec.rope_theta_global}},
            "layer_types": ["full_attention" if (gmask >> l) & 1 else "sliding_attention"
                            for l in range(spec.num_layers)],
        },
    }


def tensors_digest(tensors: dict) -> str:
    """SHA-256 over the names, dtypes, shapes and bytes of a tensor dict (sorted by name)."""
    import hashlib
    h = hashlib.sha256()
    for name in sorted(tensors):
        dtype, shape, data = tensors[name]
        h.update(f"{name}|{dtype}|{shape}|".encode())
        h.update(data)
    return h.hexdigest()


def _rand_quant(rng, name, rows, cols):
    return quant_tensors(name, *random_quant_block(rng, rows, cols))


def converter_cases() -> dict:
    """Checkpoints that pin the converter against the reference's: name -> (config, tensors,
    name prefix, shard count, converts). `converts` False marks a checkpoint both converters
    must refuse. The cases cover every name prefix the converter looks under, multi-shard
    input, full-attention layers without v, config fields left to their defaults, a layer with
    a wider FFN, an untied LM head, per-layer embeddings with shared-KV layers, and the
    Muse-Glimmer layout (untied head, attention gate, no q/k norms)."""
    import copy
    import dataclasses
    from .container import CONFIG0_TARGET

    base = CONFIG0_TARGET
    glob = dataclasses.replace(base, global_layer_mask=0b1010, global_head_dim=128, global_kv_heads=1)
    cases = {}
    cases["config0"] = (gemma4_config(base), gemma4_tensors(base, 0), "model.language_model.", 2, True)
    cases["global_layers_bare_names"] = (gemma4_config(glob), gemma4_tensors(glob, 1), "", 3, True)

    cfg = gemma4_config(base)
    del cfg["architectures"]
    for k in ("sliding_window", "final_logit_softcapping", "rope_parameters", "global_head_dim",
              "num_global_key_value_heads", "tie_word_embeddings"):
        del cfg["text_config"][k]
    cases["defaults_model_prefix"] = (cfg, gemma4_tensors(base, 2), "model.", 1, True)

    rng = np.random.default_rng(10)
    t = gemma4_tensors(base, 3)
    t.update(_rand_quant(rng, "layers.2.mlp.gate_proj", 2 * base.d_ff, base.d_model))
    t.update(_rand_quant(rng, "layers.2.mlp.up_proj", 2 * base.d_ff, base.d_model))
    t.update(_rand_quant(rng, "layers.2.mlp.down_proj", base.d_model, 2 * base.d_ff))
    cases["wide_ffn_language_model_prefix"] = (gemma4_config(base), t, "language_model.", 2, True)

    cfg = gemma4_config(base)
    cfg["text_config"]["tie_word_embeddings"] = False
    t = gemma4_tensors(base, 4)
    t.update(_rand_quant(np.random.default_rng(11), "lm_head", base.vocab_size, base.d_model))
    cases["untied_head"] = (cfg, t, "model.language_model.", 1, True)

    # Per-layer embeddings (64 wide, 512-entry table) and the last two layers sharing K/V.
    L, ple, pv, d = base.num_layers, 64, 512, base.d_model
    cfg = gemma4_config(base)
    cfg["text_config"].update(hidden_size_per_layer_input=ple, vocab_size_per_layer_input=pv, num_kv_shared_layers=2)
    t = gemma4_tensors(base, 5)
    rng = np.random.default_rng(12)
    t.update(_rand_quant(rng, "model.embed_tokens_per_layer", pv, L * ple))
    t.update(_rand_quant(rng, "model.per_layer_model_projection", L * ple, d))
    t["model.per_layer_projection_norm.weight"] = _bf16(_norm(rng, ple))
    for l in range(L):
        pre = f"layers.{l}."
        t[pre + "post_per_layer_input_norm.weight"] = _bf16(_norm(rng, d))
        t.update(_rand_quant(rng, pre + "per_layer_input_gate", ple, d))
        t.update(_rand_quant(rng, pre + "per_layer_projection", d, ple))
        if l >= L - 2:
            for n in ("self_attn.k_proj", "self_attn.v_proj"):
                for s in (".weight", ".scales", ".biases"):
                    t.pop(pre + n + s, None)
            t.pop(pre + "self_attn.k_norm.weight")
    cases["ple_shared_kv"] = (cfg, t, "model.language_model.", 2, True)

    # Muse-Glimmer: every geometry field but the layer count left to the architecture's defaults.
    rng = np.random.default_rng(13)
    t = {}
    t.update(_rand_quant(rng, "embed_tokens", 1024, d))
    t["norm.weight"] = _bf16(_norm(rng, d))
    t.update(_rand_quant(rng, "lm_head", 1024, d))
    for l in range(3):
        pre = f"layers.{l}."
        for n in ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
                  "post_feedforward_layernorm"):
            t[pre + n + ".weight"] = _bf16(_norm(rng, d))
        for n, rows, cols in (("self_attn.q_proj", 256, d), ("self_attn.k_proj", 64, d), ("self_attn.v_proj", 64, d),
                              ("self_attn.gate_proj", 256, d), ("self_attn.o_proj", d, 256),
                              ("mlp.gate_proj", 512, d), ("mlp.up_proj", 512, d), ("mlp.down_proj", d, 512)):
            t.update(_rand_quant(rng, pre + n, rows, cols))
    cfg = {"architectures": ["MuseGlimmerForConditionalGeneration"],
           "text_config": {"num_hidden_layers": 3,
                           "layer_types": ["sliding_attention", "full_attention", "sliding_attention"]}}
    cases["muse_glimmer_defaults"] = (cfg, t, "model.", 2, True)

    moe = copy.deepcopy(gemma4_config(base))
    moe["text_config"]["num_experts"] = 8
    cases["refused_moe"] = (moe, gemma4_tensors(base, 0), "model.language_model.", 1, False)
    nolt = copy.deepcopy(gemma4_config(base))
    del nolt["text_config"]["layer_types"]
    cases["refused_no_layer_types"] = (nolt, gemma4_tensors(base, 0), "model.language_model.", 1, False)
    return cases


def assistant_tensors(spec: MtpSpec, seed: int = 0, centered: bool = False) -> dict:
    """An MTP assistant's tensors, drawn as container.build_mtp_container draws: the embedding
    [V][hidden], pre_projection [hidden][2 x backbone], post_projection [backbone][hidden], the
    final norm, then per layer four [hidden] norms, q_norm, layer_scalar and q, o, gate, up, down."""
    rng = np.random.default_rng(seed)
    h, bb, I = spec.hidden, spec.backbone, spec.intermediate
    out = {}
    for name, rows, cols in (("model.embed_tokens", spec.vocab_size, h), ("pre_projection", h, 2 * bb),
                             ("post_projection", bb, h)):
        out.update(quant_tensors(name, *random_quant_block(rng, rows, cols, centered)))
    out["model.norm.weight"] = _bf16(_norm(rng, h))
    scalar = f32_to_bf16_bits(np.array([1.0 / np.sqrt(2.0 * spec.num_layers)], dtype=np.float32))
    for l in range(spec.num_layers):
        pre = f"model.layers.{l}."
        qhd = spec.q_head_dim(l)
        qd = spec.num_q_heads * qhd
        for n in ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
                  "post_feedforward_layernorm"):
            out[pre + n + ".weight"] = _bf16(_norm(rng, h))
        out[pre + "self_attn.q_norm.weight"] = _bf16(_norm(rng, qhd))
        out[pre + "layer_scalar"] = _bf16(scalar)
        for name, rows, cols in (("self_attn.q_proj", qd, h), ("self_attn.o_proj", h, qd), ("mlp.gate_proj", I, h),
                                 ("mlp.up_proj", I, h), ("mlp.down_proj", h, I)):
            out.update(quant_tensors(pre + name, *random_quant_block(rng, rows, cols, centered)))
    return out


def assistant_config(spec: MtpSpec) -> dict:
    """config.json of an MTP assistant, stating every value the .g4mtp header records."""
    return {
        "architectures": ["Gemma4AssistantForCausalLM"],
        "backbone_hidden_size": spec.backbone,
        "text_config": {
            "num_hidden_layers": spec.num_layers, "hidden_size": spec.hidden, "intermediate_size": spec.intermediate,
            "vocab_size": spec.vocab_size, "num_attention_heads": spec.num_q_heads,
            "num_key_value_heads": spec.num_kv_heads, "head_dim": spec.head_dim,
            "global_head_dim": spec.global_head_dim, "num_global_key_value_heads": spec.global_kv_heads,
            "sliding_window": spec.sliding_window,
            "layer_types": ["full_attention" if (spec.global_layer_mask >> l) & 1 else "sliding_attention"
                            for l in range(spec.num_layers)],
        },
    }


def assistant_cases() -> dict:
    """MTP assistant checkpoints that pin convert_assistant against the reference's assistant
    converter, in the converter_cases() form: the test drafter with every field stated and bare
    names; a three-layer drafter under "language_model." with its geometry and layer_types left
    to the defaults; and one missing a tensor, which both converters refuse."""
    from .container import MTP_TEST_TARGET
    spec = MtpSpec.for_target(MTP_TEST_TARGET)
    three = MtpSpec.for_target(MTP_TEST_TARGET, num_layers=3)
    under = {"language_model." + k: v for k, v in assistant_tensors(three, 21).items()}
    missing = assistant_tensors(spec, 22)
    del missing["pre_projection.biases"]
    return {
        "assistant_test_drafter": (assistant_config(spec), assistant_tensors(spec, 20), "", 2, True),
        "assistant_defaults_language_model_prefix": (
            {"backbone_hidden_size": three.backbone, "text_config": {"num_hidden_layers": 3}}, under, "", 3, True),
        "assistant_refused_missing_tensor": (assistant_config(spec), missing, "", 1, False),
    }


def e2b_tensors(spec: ModelSpec, ple_dim: int, kv_shared: int, seed: int, wide_shared_ffn: bool = False) -> dict:
    """Tensors of an E2B-style model: `spec`'s layers plus per-layer inputs of width `ple_dim`
    (the [vocab][L*ple_dim] table, its projection from the embedding and the slice norm; per layer
    the gate [ple_dim][d], the projection [d][ple_dim] and their output norm), with the last
    `kv_shared` layers reading another layer's K/V (no k/v projections, no k_norm). Every layer has
    its own v (V is the raw K only without per-layer inputs). `wide_shared_ffn` doubles the FFN
    of the shared layers, as E2B does. Zero-mean weights."""
    rng = np.random.default_rng(seed)
    d, L = spec.d_model, spec.num_layers

    def q(name, rows, cols):
        return quant_tensors(name, *random_quant_block(rng, rows, cols, True))

    out = q("embed_tokens", spec.vocab_size, d)
    out["norm.weight"] = _bf16(_norm(rng, d))
    out.update(q("model.embed_tokens_per_layer", spec.vocab_size, L * ple_dim))
    out.update(q("model.per_layer_model_projection", L * ple_dim, d))
    out["model.per_layer_projection_norm.weight"] = _bf16(_norm(rng, ple_dim))
    scalar = f32_to_bf16_bits(np.array([1.0 / np.sqrt(2.0 * L)], dtype=np.float32))
    for l in range(L):
        hd, qh, kvh, _ = spec.layer_geometry(l)
        shared = l >= L - kv_shared
        ffn = spec.d_ff * (2 if shared and wide_shared_ffn else 1)
        pre = f"layers.{l}."
        for n in ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
                  "post_feedforward_layernorm", "post_per_layer_input_norm"):
            out[pre + n + ".weight"] = _bf16(_norm(rng, d))
        out[pre + "self_attn.q_norm.weight"] = _bf16(_norm(rng, hd))
        if not shared:
            out[pre + "self_attn.k_norm.weight"] = _bf16(_norm(rng, hd))
        out[pre + "layer_scalar"] = _bf16(scalar)
        out.update(q(pre + "self_attn.q_proj", qh * hd, d))
        if not shared:
            out.update(q(pre + "self_attn.k_proj", kvh * hd, d))
            out.update(q(pre + "self_attn.v_proj", kvh * hd, d))
        out.update(q(pre + "self_attn.o_proj", d, qh * hd))
        out.update(q(pre + "mlp.gate_proj", ffn, d))
        out.update(q(pre + "mlp.up_proj", ffn, d))
        out.update(q(pre + "mlp.down_proj", d, ffn))
        out.update(q(pre + "per_layer_input_gate", ple_dim, d))
        out.update(q(pre + "per_layer_projection", d, ple_dim))
    return out


def forward_cases() -> dict:
    """Checkpoints on which the reference's independent NumPy forward pass
    (tools/numpy_reference.py) pins converter + oracle: name -> (config, tensors, prompt ids).
    Zero-mean ("centered") weights, vocabulary 1024 to keep the committed logits small, names
    under "model." as that tool reads them. The cases: the config-0 shape; full-attention layers
    (head_dim 128, rotating all 64 pairs, which a partial_rotary_factor of 1.0 tells the NumPy
    pass); the same with a 4-key sliding window that the prompt wraps twice; and head_dim-512
    full-attention layers with GQA 2, on the default factor of 0.25 (64 of 256 pairs)."""
    import dataclasses
    from .container import CONFIG0_TARGET

    base = dataclasses.replace(CONFIG0_TARGET, vocab_size=1024)
    glob = dataclasses.replace(base, global_layer_mask=0b1010, global_head_dim=128, global_kv_heads=1)
    wide = dataclasses.replace(base, num_kv_heads=2, global_layer_mask=0b0100, global_head_dim=512,
                               global_kv_heads=1)
    cases = {}
    for name, spec, seed, prompt, prf in (
            ("config0_shape", base, 30, [2, 105, 17, 900, 1023, 3], None),
            ("global_layers", glob, 31, [2, 7, 300, 1000, 55, 9], 1.0),
            ("window_wrap", dataclasses.replace(glob, sliding_window=4), 32, [2, 7, 300, 1000, 55, 9, 77, 512, 4], 1.0),
            ("global_hd512_gqa2", wide, 33, [2, 640, 31, 8, 999, 100], None)):
        cfg = gemma4_config(spec)
        if prf is not None:
            cfg["text_config"]["rope_parameters"]["full_attention"]["partial_rotary_factor"] = prf
        cases[name] = (cfg, gemma4_tensors(spec, seed, centered=True), prompt)
    # E2B-style: per-layer inputs 64 wide and the last two layers sharing K/V. The first is all
    # sliding with double-wide FFNs on the shared layers; the second alternates sliding and
    # full-attention layers, so each shared layer takes its own type's donor (layers 2 and 3).
    six = dataclasses.replace(glob, num_layers=6, global_layer_mask=0b101010)
    for name, spec, seed, prompt, prf, wide in (
            ("e2b_ple_shared_kv", base, 34, [2, 686, 824, 23, 827, 480], None, True),
            ("e2b_ple_shared_kv_global", six, 35, [2, 90, 1, 333, 812, 64, 7], 1.0, False)):
        cfg = gemma4_config(spec)
        cfg["text_config"].update(hidden_size_per_layer_input=64, vocab_size_per_layer_input=spec.vocab_size,
                                  num_kv_shared_layers=2)
        if prf is not None:
            cfg["text_config"]["rope_parameters"]["full_attention"]["partial_rotary_factor"] = prf
        cases[name] = (cfg, e2b_tensors(spec, 64, 2, seed, wide_shared_ffn=wide), prompt)
    return cases


def write_checkpoint(directory, config: dict, tensors: dict, prefix: str = "model.language_model.",
                     shards: int = 1) -> Path:
    """Writes config.json and the tensors as `shards` safetensors files (round-robin by name),
    each tensor name under `prefix` unless it already starts with "model.". Returns the directory."""
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    (directory / "config.json").write_text(json.dumps(config, indent=1), encoding="utf-8")
    names = sorted(tensors)
    for s in range(shards):
        header, blobs, off = {"__metadata__": {"format": "mlx"}}, [], 0
        for name in names[s::shards]:
            dtype, shape, data = tensors[name]
            key = name if name.startswith("model.") else prefix + name
            header[key] = {"dtype": dtype, "shape": shape, "data_offsets": [off, off + len(data)]}
            blobs.append(data)
            off += len(data)
        meta = json.dumps(header, separators=(",", ":")).encode("utf-8")
        meta += b" " * ((-len(meta)) % 8)
        with open(directory / f"model-{s + 1:05d}-of-{shards:05d}.safetensors", "wb") as f:
            f.write(struct.pack("<Q", len(meta)))
            f.write(meta)
            for b in blobs:
                f.write(b)
    return directory
