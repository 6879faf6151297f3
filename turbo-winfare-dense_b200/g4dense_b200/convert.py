"""Hugging Face / MLX checkpoint -> `.g4dense` v3 container, the engine's input format.

The checkpoint is a directory with config.json and *.safetensors shards holding MLX-style INT4
group-64 affine weights (`<name>.weight` as packed uint32 nibble words, `<name>.scales` and
`<name>.biases` as bf16) and bf16 norms -- what tools/convert_hf_to_g4dense.py of the reference
reads. The output is the container that tool writes (include/g4dense/format.hpp:26-110), byte for
byte:

* a 4096-byte header;
* the embedding block: the embedding's packed weight, scales and biases, then the final norm;
* the LM-head block (weight, scales, biases) when the head is untied (Muse-Glimmer);
* the per-layer-embedding block when `hidden_size_per_layer_input` is set (E2B/E4B);
* one block per layer: the bf16 norms (input, post-attention, pre-FFN, post-FFN; for Gemma-4
  also q_norm, k_norm unless the layer reuses another layer's K/V, and `layer_scalar`; the
  per-layer-input norm with per-layer embeddings), then the projections q, k, v, (Muse: the
  attention gate), o, gate, up, down (and the two per-layer-input projections), each starting on
  a 16-byte boundary of its block. A Gemma-4 layer without its own v (a full-attention layer
  whose V is its raw K) skips it; a shared-KV layer has no k, v or k_norm.

Every block is zero-padded to 4096 bytes and the header holds the payload's SHA-256.

Tensors are looked up as the reference does (the bare name, then under "model.",
"language_model." and "model.language_model."), and config.json fields take the same
per-architecture defaults, so a checkpoint becomes the same container. Tensor bytes are copied
from the shards in chunks of at most 64 MiB and hashed on the way; the header is written last. The
converter's memory use is bounded by one chunk, whatever the checkpoint's size.

The engine itself runs Gemma-4 dense models without per-layer embeddings or shared KV; its loader
rejects the other containers with the reason (validate_header). Mixture-of-experts checkpoints are
refused here, as the reference refuses them.

The MTP assistant drafter's checkpoint converts to a `.g4mtp` container the same way
(convert_assistant, tools/convert_hf_assistant.py of the reference).

    python -m g4dense_b200.convert --input CHECKPOINT_DIR --out model.g4dense
    python -m g4dense_b200.convert --assistant --input ASSISTANT_DIR --out assistant.g4mtp
"""
from __future__ import annotations

import argparse
import hashlib
import json
import struct
import sys
from pathlib import Path

from .container import (ALIGNMENT, GROUP, HEADER_FMT, HEADER_SIZE, MAGIC, MTP_HEADER_FMT, MTP_MAGIC, MTP_MAX_LAYERS,
                        MTP_VERSION, QUANT_AFFINE_INT4_G64, VERSION)

MAX_LAYERS = 60
_PREFIXES = ("", "model.", "language_model.", "model.language_model.")
_MUSE_ARCHS = ("MuseGlimmerForConditionalGeneration", "MuseForConditionalGeneration")

# config.json key -> (Gemma-4 default, Muse-Glimmer default): the defaults the reference's
# converter applies when a key is absent (tools/convert_hf_to_g4dense.py:57-73).
_DEFAULTS = {
    "num_hidden_layers": (60, 52), "hidden_size": (5376, 6656), "intermediate_size": (21504, 19968),
    "num_attention_heads": (32, 32), "num_key_value_heads": (16, 2), "head_dim": (256, 128),
    "vocab_size": (262144, 202048), "sliding_window": (1024, 2048), "final_logit_softcapping": (30.0, 20.0),
    "qk_scale_factor": (1.0, 3.87), "output_multiplier": (1.0, 0.196116),
}
_ROPE_DEFAULTS = {"sliding_attention": (10000.0, 500000.0), "full_attention": (1000000.0, 0.0)}


class CheckpointError(ValueError):
    pass


class _Span:
    """One tensor's bytes inside a shard; copied out in chunks of at most 64 MiB."""

    CHUNK = 64 << 20

    def __init__(self, key: str, path: Path, offset: int, length: int):
        self.key, self.path, self.offset, self.length = key, path, offset, length

    def __len__(self) -> int:
        return self.length

    def chunks(self):
        with open(self.path, "rb") as f:
            f.seek(self.offset)
            left = self.length
            while left:
                data = f.read(min(left, self.CHUNK))
                if not data:
                    raise CheckpointError(f"tensor {self.key}: shard {self.path} ends early")
                left -= len(data)
                yield data


class _Tensors:
    """The tensors of every shard: name -> (file, absolute byte offset, byte length, shape).
    A name is looked up under each of `prefixes` in turn."""

    def __init__(self, directory: Path, prefixes=_PREFIXES):
        self.where = {}
        self.prefixes = prefixes
        shards = sorted(directory.glob("*.safetensors"))
        if not shards:
            raise CheckpointError(f"no .safetensors shards in {directory}")
        for shard in shards:
            size = shard.stat().st_size
            with open(shard, "rb") as f:
                raw = f.read(8)
                if len(raw) != 8:
                    raise CheckpointError(f"{shard}: not a safetensors file")
                (n,) = struct.unpack("<Q", raw)
                meta = json.loads(f.read(n).decode("utf-8"))
            for name, info in meta.items():
                if name == "__metadata__":
                    continue
                lo, hi = info["data_offsets"]
                if not 0 <= lo <= hi or 8 + n + hi > size:
                    raise CheckpointError(f"tensor {name}: bytes {lo}..{hi} lie outside shard {shard}")
                self.where[name] = (shard, 8 + n + lo, hi - lo, info["shape"])

    def key(self, name):
        for p in self.prefixes:
            if p + name in self.where:
                return p + name
        return None

    def has(self, name):
        return self.key(name) is not None

    def shape(self, name):
        k = self.key(name)
        return None if k is None else self.where[k][3]

    def read(self, name, optional=False):
        """The tensor's bytes as a _Span (b"" for a missing optional tensor)."""
        k = self.key(name)
        if k is None:
            if optional:
                return b""
            raise CheckpointError(f"tensor {name} is not in the checkpoint")
        path, off, length, _ = self.where[k]
        return _Span(k, path, off, length)

    def quantized(self, name, scales_optional=True):
        """[packed weight, scales, biases] of one quantized matrix; missing scales/biases are empty."""
        return [self.read(name + ".weight"), self.read(name + ".scales", scales_optional),
                self.read(name + ".biases", scales_optional)]


def geometry(config: dict) -> dict:
    """The header's model fields from config.json (its text_config when present)."""
    arch = (config.get("architectures") or ["Gemma4ForConditionalGeneration"])[0]
    muse = arch in _MUSE_ARCHS or config.get("model_type") == "muse_glimmer"
    t = config.get("text_config", config)
    if t.get("moe_layers") or t.get("num_experts"):
        raise CheckpointError("unsupported architecture: the checkpoint declares mixture-of-experts blocks; "
                              "this engine runs dense models")
    pick = lambda key: t.get(key, _DEFAULTS[key][muse])  # noqa: E731
    g = {
        "muse": muse,
        "layers": int(pick("num_hidden_layers")),
        "d_model": int(pick("hidden_size")),
        "d_ff": int(pick("intermediate_size")),
        "q_heads": int(pick("num_attention_heads")),
        "kv_heads": int(pick("num_key_value_heads")),
        "head_dim": int(pick("head_dim")),
        "vocab": int(pick("vocab_size")),
        "window": int(pick("sliding_window")),
        "softcap": float(pick("final_logit_softcapping")),
        "qk_scale": float(pick("qk_scale_factor")),
        "out_mult": float(pick("output_multiplier")),
        "tied": not muse and bool(t.get("tie_word_embeddings", True)),
        "ple_dim": int(t.get("hidden_size_per_layer_input", 0) or 0),
        "ple_vocab": int(t.get("vocab_size_per_layer_input", 0) or 0),
        "kv_shared": int(t.get("num_kv_shared_layers", 0) or 0),
    }
    g["attn_out_dim"] = g["q_heads"] * g["head_dim"] if muse else g["d_model"]
    g["global_head_dim"] = g["head_dim"] if muse else int(t.get("global_head_dim", 512))
    gkv = t.get("num_global_key_value_heads")
    g["global_kv_heads"] = int(gkv) if gkv else g["kv_heads"]
    rope = t.get("rope_parameters", {})
    for kind, field in (("sliding_attention", "theta_local"), ("full_attention", "theta_global")):
        g[field] = float(rope.get(kind, {}).get("rope_theta", _ROPE_DEFAULTS[kind][muse]))
    layer_types = t.get("layer_types") or []
    if not layer_types:
        raise CheckpointError("config.json has no layer_types")
    if g["layers"] > MAX_LAYERS or len(layer_types) < g["layers"]:
        raise CheckpointError(f"{g['layers']} layers with {len(layer_types)} layer_types: the container holds at "
                              f"most {MAX_LAYERS} layers, each with its layer_type")
    g["global"] = [lt == "full_attention" for lt in layer_types[:g["layers"]]]
    g["mask"] = sum(1 << i for i, lt in enumerate(layer_types[:64]) if lt == "full_attention")
    g["first_shared"] = g["layers"] - g["kv_shared"] if g["kv_shared"] else g["layers"]
    return g


def _layer_tensors(g: dict, l: int):
    """Layer l's block in file order: ("norm", name) entries, then ("proj", name, optional)."""
    shared = l >= g["first_shared"]
    out = [("norm", n) for n in ("input_layernorm.weight", "post_attention_layernorm.weight",
                                 "pre_feedforward_layernorm.weight", "post_feedforward_layernorm.weight")]
    if not g["muse"]:
        out.append(("norm", "self_attn.q_norm.weight"))
        if not shared:
            out.append(("norm", "self_attn.k_norm.weight"))
        out.append(("norm", "layer_scalar"))
    if g["ple_dim"]:
        out.append(("norm", "post_per_layer_input_norm.weight"))
    out.append(("proj", "self_attn.q_proj", False))
    if not shared:
        out += [("proj", "self_attn.k_proj", False), ("proj", "self_attn.v_proj", not g["muse"])]
    if g["muse"]:
        out.append(("proj", "self_attn.gate_proj", False))
    out += [("proj", n, False) for n in ("self_attn.o_proj", "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj")]
    if g["ple_dim"]:
        out += [("proj", "per_layer_input_gate", False), ("proj", "per_layer_projection", False)]
    return out


def _run(input_dir, output_path, geometry_of, write, prefixes) -> Path:
    """Reads config.json and the shard index of `input_dir`, then writes the container through a
    temporary name that is renamed when complete and removed when the conversion fails."""
    src = Path(input_dir)
    cfg_path = src / "config.json"
    if not cfg_path.exists():
        raise CheckpointError(f"no config.json in {src}")
    g = geometry_of(json.loads(cfg_path.read_text(encoding="utf-8")))
    T = _Tensors(src, prefixes)
    out = Path(output_path)
    out.parent.mkdir(parents=True, exist_ok=True)
    tmp = out.with_suffix(out.suffix + ".tmp")
    try:
        write(T, g, tmp)
    except BaseException:
        tmp.unlink(missing_ok=True)
        raise
    tmp.replace(out)
    return out


def convert(input_dir, output_path) -> Path:
    """Writes the .g4dense container for the model checkpoint in `input_dir` to `output_path`."""
    return _run(input_dir, output_path, geometry, _write, _PREFIXES)


class _BlockWriter:
    """Streams 4096-aligned blocks behind a zeroed header and hashes them as they go."""

    def __init__(self, f):
        self.f, self.sha = f, hashlib.sha256()
        f.write(b"\x00" * HEADER_SIZE)

    def __call__(self, parts) -> int:
        """Writes one block (byte strings and tensor spans), zero-padded to the container
        alignment; returns its size."""
        n = 0
        for part in parts:
            for b in (part.chunks() if isinstance(part, _Span) else (part,)):
                self.f.write(b)
                self.sha.update(b)
            n += len(part)
        tail = b"\x00" * ((-n) % ALIGNMENT)
        self.f.write(tail)
        self.sha.update(tail)
        return n + len(tail)

    def header(self, raw: bytes) -> None:
        assert len(raw) == HEADER_SIZE
        self.f.seek(0)
        self.f.write(raw)


def _layer_parts(T: _Tensors, pre: str, norms, projections) -> list:
    """One layer's tensors in file order: the norms back to back, then each projection's
    packed weight, scales and biases starting on a 16-byte boundary of the block."""
    parts, n = [], 0
    for name in norms:
        parts.append(T.read(pre + name))
        n += len(parts[-1])
    for name in projections:
        data = [b"\x00" * ((-n) % 16)] + T.quantized(pre + name)
        parts += data
        n += sum(len(x) for x in data)
    return parts


def _write(T: _Tensors, g: dict, path: Path) -> None:
    """Streams the blocks to `path` behind a zeroed header, then writes the header."""
    with open(path, "wb") as f:
        block = _BlockWriter(f)
        embed_size = block(T.quantized("embed_tokens") + [T.read("norm.weight")])
        head_size = 0 if g["tied"] else block(T.quantized("lm_head"))
        ple_size = 0
        if g["ple_dim"]:
            ple_size = block(T.quantized("model.embed_tokens_per_layer", False) +
                             T.quantized("model.per_layer_model_projection", False) +
                             [T.read("model.per_layer_projection_norm.weight")])
        layer_sizes, layer_d_ff = [], []
        for l in range(g["layers"]):
            pre = f"layers.{l}."
            entries = _layer_tensors(g, l)
            norms = [e[1] for e in entries if e[0] == "norm"]
            projections = [e[1] for e in entries
                           if e[0] == "proj" and not (e[2] and not T.has(pre + e[1] + ".weight"))]
            shape = T.shape(pre + "mlp.gate_proj.weight")
            layer_d_ff.append(int(shape[0]) if shape else g["d_ff"])
            layer_sizes.append(block(_layer_parts(T, pre, norms, projections)))

        head_offset = HEADER_SIZE if g["tied"] else HEADER_SIZE + embed_size
        cur = HEADER_SIZE + embed_size + head_size
        ple_offset = cur if ple_size else 0
        cur += ple_size
        layer_offsets = []
        for n in layer_sizes:
            layer_offsets.append(cur)
            cur += n
        pad60 = lambda v: list(v) + [0] * (MAX_LAYERS - len(v))  # noqa: E731
        header = struct.pack(
            HEADER_FMT, MAGIC, VERSION, QUANT_AFFINE_INT4_G64, g["layers"], g["d_model"], g["d_ff"], g["q_heads"],
            g["kv_heads"], g["head_dim"], g["vocab"], g["window"], GROUP, 1, int(g["tied"]), g["mask"],
            g["theta_local"], g["theta_global"], 1.0, g["softcap"], HEADER_SIZE, embed_size, head_offset,
            embed_size if g["tied"] else head_size, *pad60(layer_offsets), *pad60(layer_sizes), block.sha.digest(),
            g["global_head_dim"], g["global_kv_heads"], g["ple_dim"], g["ple_vocab"], g["kv_shared"], 0, ple_offset,
            ple_size, *pad60(layer_d_ff), int(g["muse"]), g["attn_out_dim"], g["qk_scale"], g["out_mult"],
            b"\x00" * 2696)
        block.header(header)


# ------------------------------------------------------------------ .g4mtp (the MTP assistant)

# The assistant's config.json defaults (tools/convert_hf_assistant.py:49-62): the Gemma-4 31B
# assistant's geometry.
_ASSISTANT_DEFAULTS = {
    "num_hidden_layers": 4, "hidden_size": 1024, "intermediate_size": 8192, "vocab_size": 262144,
    "num_attention_heads": 32, "num_key_value_heads": 16, "head_dim": 256, "global_head_dim": 512,
    "num_global_key_value_heads": 4, "sliding_window": 1024,
}
_ASSISTANT_PREFIXES = ("", "language_model.")
_ASSISTANT_NORMS = ("input_layernorm.weight", "post_attention_layernorm.weight", "pre_feedforward_layernorm.weight",
                    "post_feedforward_layernorm.weight", "self_attn.q_norm.weight", "layer_scalar")
_ASSISTANT_PROJECTIONS = ("self_attn.q_proj", "self_attn.o_proj", "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj")


def assistant_geometry(config: dict) -> dict:
    """The .g4mtp header's model fields. `backbone_hidden_size` (the target's width) is read
    from the top level of config.json, the rest from its text_config when present; layer_types
    defaults to sliding layers with a full-attention last layer."""
    t = config.get("text_config", config)
    g = {k: int(t.get(k, v)) for k, v in _ASSISTANT_DEFAULTS.items()}
    g["backbone"] = int(config.get("backbone_hidden_size", 5376))
    L = g["num_hidden_layers"]
    if not 1 <= L <= MTP_MAX_LAYERS:
        raise CheckpointError(f"{L} assistant layers: the .g4mtp container holds 1..{MTP_MAX_LAYERS}")
    layer_types = t.get("layer_types", ["sliding_attention"] * (L - 1) + ["full_attention"])
    g["mask"] = sum(1 << i for i, lt in enumerate(layer_types) if lt == "full_attention")
    return g


def _write_assistant(T: _Tensors, g: dict, path: Path) -> None:
    with open(path, "wb") as f:
        block = _BlockWriter(f)
        sections = [block(T.quantized("model.embed_tokens", False)),  # the tied LM head too
                    block(T.quantized("pre_projection", False)),       # [hidden][2 x backbone]
                    block(T.quantized("post_projection", False)),      # [backbone][hidden]
                    block([T.read("model.norm.weight")])]
        layer_sizes = [block(_layer_parts(T, f"model.layers.{l}.", _ASSISTANT_NORMS, _ASSISTANT_PROJECTIONS))
                       for l in range(g["num_hidden_layers"])]
        spans, cur = [], HEADER_SIZE
        for n in sections + layer_sizes:
            spans.append((cur, n))
            cur += n
        pad8 = lambda v: list(v) + [0] * (MTP_MAX_LAYERS - len(v))  # noqa: E731
        block.header(struct.pack(
            MTP_HEADER_FMT, MTP_MAGIC, MTP_VERSION, QUANT_AFFINE_INT4_G64, g["num_hidden_layers"], g["backbone"],
            g["hidden_size"], g["intermediate_size"], g["vocab_size"], g["num_attention_heads"],
            g["num_key_value_heads"], g["head_dim"], g["global_head_dim"], g["num_global_key_value_heads"],
            g["sliding_window"], g["mask"], GROUP, 1, *[v for span in spans[:4] for v in span],
            *pad8([o for o, _ in spans[4:]]), *pad8([n for _, n in spans[4:]]), block.sha.digest(), b"\x00" * 3800))


def convert_assistant(input_dir, output_path) -> Path:
    """Writes the .g4mtp container for the MTP assistant checkpoint in `input_dir` to
    `output_path`, byte for byte the container tools/convert_hf_assistant.py writes: the embedding
    (tied LM head), pre-projection, post-projection and final-norm sections, then per layer the
    four norms, q_norm and layer_scalar, then q, o, gate, up, down on 16-byte boundaries (the
    assistant reads its K/V from the target's cache, so it has no k, v or k_norm). Names are looked
    up bare and under "language_model."."""
    return _run(input_dir, output_path, assistant_geometry, _write_assistant, _ASSISTANT_PREFIXES)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="Convert an MLX INT4 Gemma-4 checkpoint to a .g4dense container, "
                                             "or its MTP assistant to a .g4mtp container")
    ap.add_argument("--input", "--input-dir", dest="input", required=True,
                    help="checkpoint directory (config.json + *.safetensors)")
    ap.add_argument("--out", "--output-file", dest="out", required=True, help="output container path")
    ap.add_argument("--assistant", action="store_true", help="the checkpoint is an MTP assistant: write .g4mtp")
    a = ap.parse_args(argv)
    try:
        path = (convert_assistant if a.assistant else convert)(a.input, a.out)
    except (CheckpointError, OSError, KeyError, ValueError) as e:
        print(f"convert: {e}", file=sys.stderr)
        return 1
    print(f"wrote {path} ({path.stat().st_size:,} bytes)")
    return 0


if __name__ == "__main__":
    sys.exit(main())
