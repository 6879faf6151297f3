"""Synthetic `.g4dense` v3 container writer and header reader.

The on-disk contract is the reference's: a 4096-byte packed ``G4DenseHeader``
(include/g4dense/format.hpp:26-110) followed by 4096-aligned blocks.

* Embedding block (src/cpu_reference.cpp:260-285, 610-614): packed INT4 words
  ``[V][d/8]`` u32 (nibble c%8 of word c/8 at bits 4*(c%8), low nibble first), bf16
  scales ``[V][d/64]``, bf16 biases ``[V][d/64]``, then the bf16 final-norm weight
  ``[d]``. The LM head is tied: ``lm_head_offset == embed_offset``
  (tools/make_synthetic_model.py:189-191).
* Layer block (src/cpu_reference.cpp:324-395, src/runner.cpp:271-370): bf16 norms
  in, post-attn, pre-FFN, post-FFN (each ``[d]``), q_norm and k_norm (each
  ``[head_dim]`` of that layer's geometry), one bf16 ``layer_scalar``; then for each
  of q, k, v (absent on global layers), o, gate, up, down: zero-pad to a 16-byte
  boundary relative to the layer start, then W, scales, biases.

Value distributions are BASELINE config 0's, drawn from ``numpy.random.default_rng(seed)``
in this fixed order: embedding (nibble bytes, scales, biases), final norm, then per layer
the six norms in file order, then per projection (nibble bytes, scales, biases).
Nibbles are uniform in 0..15 (uniform random bytes), scales are |N(0, 0.02)|, biases
N(0, 0.01), norm weights 1 + N(0, 0.05); all non-quantized values are rounded to bf16
(round-to-nearest-even). ``layer_scalar`` is 1/sqrt(2L) as in
tools/make_synthetic_model.py:143. Embeddings are INT4 because the format has no bf16
embedding block.
"""
from __future__ import annotations

import dataclasses
import hashlib
import struct
from pathlib import Path

import numpy as np

HEADER_SIZE = 4096
ALIGNMENT = 4096
MAGIC = 0x4734444E
VERSION = 3
QUANT_AFFINE_INT4_G64 = 1
GROUP = 64
# The packed header layout of G4DenseHeader (include/g4dense/format.hpp:26-110).
HEADER_FMT = "<IIIIIIIIIIIIIIQffffQQQQ60Q60Q32sIIIIIIQQ60IIIff2696s"
assert struct.calcsize(HEADER_FMT) == HEADER_SIZE


@dataclasses.dataclass
class ModelSpec:
    num_layers: int
    d_model: int
    d_ff: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    vocab_size: int
    sliding_window: int = 1024
    global_layer_mask: int = 0
    global_head_dim: int = 0
    global_kv_heads: int = 0
    rope_theta_local: float = 10000.0
    rope_theta_global: float = 1000000.0
    softcap: float = 30.0

    def layer_geometry(self, l: int):
        """(head_dim, q_heads, kv_heads, is_global) -- resolve_layer_geometry,
        include/g4dense/format.hpp:229-241."""
        is_global = bool((self.global_layer_mask >> l) & 1)
        hd, kvh = self.head_dim, self.num_kv_heads
        if is_global:
            hd = self.global_head_dim or 512
            kvh = self.global_kv_heads or 4
        return hd, self.num_q_heads, kvh, is_global

    def layer_projections(self, l: int):
        """[(name, rows, cols)] in file order (src/cpu_reference.cpp:383-395)."""
        hd, qh, kvh, is_global = self.layer_geometry(l)
        d, f = self.d_model, self.d_ff
        out = [("q", qh * hd, d), ("k", kvh * hd, d)]
        if not is_global:
            out.append(("v", kvh * hd, d))
        out += [("o", d, qh * hd), ("gate", f, d), ("up", f, d), ("down", d, f)]
        return out


# the tiny target / drafter pair.
CONFIG0_TARGET = ModelSpec(num_layers=4, d_model=256, d_ff=1024, num_q_heads=4, num_kv_heads=1,
                           head_dim=64, vocab_size=4096)
CONFIG0_DRAFT = ModelSpec(num_layers=2, d_model=128, d_ff=512, num_q_heads=2, num_kv_heads=1,
                          head_dim=64, vocab_size=4096)
# Gemma-4-31B shape (docs/FORWARD_PASS.md constants): global layers every 6th from 5.
GEMMA4_31B = ModelSpec(num_layers=60, d_model=5376, d_ff=21504, num_q_heads=32, num_kv_heads=16,
                       head_dim=256, vocab_size=262144, sliding_window=1024,
                       global_layer_mask=0x0820820820820820, global_head_dim=512, global_kv_heads=4)
# Two layers of the 31B at full width (one sliding, one global) with the full 262144-row embedding
# and LM head: the CPU-baseline sample and the full-shape parity case.
GEMMA4_31B_TWO_LAYERS = dataclasses.replace(GEMMA4_31B, num_layers=2, global_layer_mask=0b10)
# Gemma-4-E2B-shaped drafter used by BASELINE config 3 (no PLE, no KV sharing).
E2B_DRAFT = ModelSpec(num_layers=35, d_model=1536, d_ff=6144, num_q_heads=8, num_kv_heads=1,
                      head_dim=256, vocab_size=262144, sliding_window=512)


# A mid-size drafter (a test aid): d 512 (four k-tiles per projection), FFN 2048, GQA 4 over two KV
# heads of 128 and a 64-key window that 200 chained steps wrap, at a size the CPU oracle runs in
# seconds.
MID_TEST_DRAFT = ModelSpec(num_layers=3, d_model=512, d_ff=2048, num_q_heads=8, num_kv_heads=2, head_dim=128,
                             vocab_size=4096, sliding_window=64)


# Gemma-4-31B attention geometry at toy width (a test aid): sliding layers with head_dim 256 and
# GQA 2 over a 48-key window (the KV ring wraps), one full-attention layer with head_dim 512, a
# single KV head (GQA 4) and V taken from the raw K.
GEOM31_TEST = ModelSpec(num_layers=3, d_model=256, d_ff=512, num_q_heads=4, num_kv_heads=2, head_dim=256,
                        vocab_size=4096, sliding_window=48, global_layer_mask=0b010, global_head_dim=512,
                        global_kv_heads=1)

# Tensor-parallel test geometry at config-0 scale (a test aid): 8 query heads and 8 KV heads on
# the sliding layers split evenly at TP 2/4/8; the full-attention layer (head_dim 128) has 2 KV
# heads, so TP = 8 replicates them as the 31B's four-head global layers are replicated at TP = 8.
# A 64-key window, wrapped by long prompts.
TP_TEST_TARGET = ModelSpec(num_layers=4, d_model=256, d_ff=1024, num_q_heads=8, num_kv_heads=8, head_dim=64,
                           vocab_size=4096, sliding_window=64, global_layer_mask=0b0100, global_head_dim=128,
                           global_kv_heads=2)

# Config-0 decode cases whose oracle greedy streams have no near-tie: prompt seeds found by
# scanning the oracle's top-2 margins (seeds 100.. in order) on the zero-mean ("centered")
# config-0 target (seed 0) and drafter (seed 1). Along each stream every target margin is at
# least 0.09 and every drafter margin at least 0.02, above the FP16 K/V rounding noise of the
# GPU-vs-CPU comparison, so streams and round records can be compared exactly.
PINNED_PROMPT_SEED, PINNED_PROMPT_LEN, PINNED_TOKENS = 158, 32, 64
PINNED_LONG_PROMPT_SEED, PINNED_LONG_PROMPT_LEN, PINNED_LONG_TOKENS = 114, 300, 32
# The drafter of the sampled-decoding parity cases: the BASELINE-distribution config-0 target with
# 20% of its embedding nibbles re-drawn (perturbed_copy), so rejection sampling both accepts and
# rejects drafts.
NEAR_DRAFT_EMBED_FRAC, NEAR_DRAFT_SEED = 0.2, 7
SAMPLED_PARAMS = (0.8, 0.95, 64, 5)  # temperature, top_p, top_k, seed


# The same for TP_TEST_TARGET (zero-mean, seed TP_TEST_SEED): (prompt seed, prompt length, tokens).
# Target margins along the streams are at least 0.10, the config-0 drafter's at least 0.03.
TP_TEST_SEED = 3
TP_PINNED = (137, 32, 64)
TP_PINNED_LONG = (132, 300, 32)


def tp_pinned_prompt(long: bool = False) -> np.ndarray:
    seed, n, _ = TP_PINNED_LONG if long else TP_PINNED
    return np.random.default_rng(seed).integers(0, 4096, n)


def pinned_prompt(long: bool = False) -> np.ndarray:
    if long:
        return np.random.default_rng(PINNED_LONG_PROMPT_SEED).integers(0, 4096, PINNED_LONG_PROMPT_LEN)
    return np.random.default_rng(PINNED_PROMPT_SEED).integers(0, 4096, PINNED_PROMPT_LEN)


# A target with both layer kinds at config-0 scale: the MTP drafter's tests need a sliding and a
# full-attention donor layer (the 31B's last two layers play that part for its assistant).
MTP_TEST_TARGET = ModelSpec(num_layers=4, d_model=256, d_ff=1024, num_q_heads=4, num_kv_heads=2,
                            head_dim=64, vocab_size=4096, sliding_window=64, global_layer_mask=0b1000,
                            global_head_dim=128, global_kv_heads=1)


# ---------------------------------------------------------------- .g4mtp (MTP assistant drafter)

MTP_MAGIC = 0x47344D54  # 'G4MT'
MTP_VERSION = 1
MTP_MAX_LAYERS = 8
# G4MtpHeader, include/g4dense/format.hpp:143-180 (packed, 4096 bytes).
MTP_HEADER_FMT = "<14IQ2I8Q8Q8Q32s3800s"


@dataclasses.dataclass
class MtpSpec:
    """Geometry of a Gemma-4 "assistant" MTP drafter (.g4mtp). The attention geometry must equal
    its target's donor layers: num_kv_heads/head_dim those of the target's sliding layers,
    global_kv_heads/global_head_dim those of its full-attention layers."""
    num_layers: int
    backbone: int          # the target's d_model
    hidden: int
    intermediate: int
    vocab_size: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    global_head_dim: int
    global_kv_heads: int
    sliding_window: int = 1024
    global_layer_mask: int = 0

    @classmethod
    def for_target(cls, t: ModelSpec, num_layers=4, hidden=128, intermediate=512, num_q_heads=4, global_mask=None):
        return cls(num_layers=num_layers, backbone=t.d_model, hidden=hidden, intermediate=intermediate,
                   vocab_size=t.vocab_size, num_q_heads=num_q_heads, num_kv_heads=t.num_kv_heads,
                   head_dim=t.head_dim, global_head_dim=t.global_head_dim or 512,
                   global_kv_heads=t.global_kv_heads or 4, sliding_window=t.sliding_window,
                   global_layer_mask=(1 << (num_layers - 1)) if global_mask is None else global_mask)

    def q_head_dim(self, l: int) -> int:
        return self.global_head_dim if (self.global_layer_mask >> l) & 1 else self.head_dim


# The 31B's assistant (tools/convert_hf_assistant.py:49-66 defaults): 4 layers, the last one
# full-attention.
GEMMA4_31B_ASSISTANT = MtpSpec(num_layers=4, backbone=5376, hidden=1024, intermediate=8192, vocab_size=262144,
                               num_q_heads=32, num_kv_heads=16, head_dim=256, global_head_dim=512,
                               global_kv_heads=4, sliding_window=1024, global_layer_mask=0b1000)


def build_mtp_container(spec: MtpSpec, seed: int = 0, centered: bool = False) -> bytes:
    """Full .g4mtp bytes: header, embedding (tied LM head) [V][hidden], pre-projection
    [hidden][2*backbone], post-projection [backbone][hidden], final norm [hidden], then the layers
    (tools/convert_hf_assistant.py:114-176; per-layer layout of src/mtp_runner.cpp:175-234: four
    [hidden] norms, q_norm [q_head_dim], layer_scalar, then q, o, gate, up, down, each 16-byte
    aligned). Every section is padded to 4096 bytes."""
    rng = np.random.default_rng(seed)
    h, bb, I, V = spec.hidden, spec.backbone, spec.intermediate, spec.vocab_size

    def block(rows, cols):
        p, s_, b_ = random_quant_block(rng, rows, cols, centered)
        return p.tobytes() + s_.tobytes() + b_.tobytes()

    sections = []
    for rows, cols in [(V, h), (h, 2 * bb), (bb, h)]:
        sec = bytearray(block(rows, cols))
        _pad(sec, ALIGNMENT)
        sections.append(bytes(sec))
    norm = bytearray(_norm(rng, h).tobytes())
    _pad(norm, ALIGNMENT)
    sections.append(bytes(norm))
    scalar = f32_to_bf16_bits(np.array([1.0 / np.sqrt(2.0 * spec.num_layers)], dtype=np.float32))
    layers = []
    for l in range(spec.num_layers):
        qhd = spec.q_head_dim(l)
        qd = spec.num_q_heads * qhd
        ld = bytearray()
        for _ in range(4):
            ld += _norm(rng, h).tobytes()
        ld += _norm(rng, qhd).tobytes()
        ld += scalar.tobytes()
        for rows, cols in [(qd, h), (h, qd), (I, h), (I, h), (h, I)]:
            _pad(ld, 16)
            ld += block(rows, cols)
        _pad(ld, ALIGNMENT)
        layers.append(bytes(ld))
    offs, cur = [], HEADER_SIZE
    for sec in sections:
        offs.append((cur, len(sec)))
        cur += len(sec)
    lo, ls = [0] * MTP_MAX_LAYERS, [0] * MTP_MAX_LAYERS
    for l, ld in enumerate(layers):
        lo[l], ls[l] = cur, len(ld)
        cur += len(ld)
    payload = b"".join(sections) + b"".join(layers)
    header = struct.pack(
        MTP_HEADER_FMT, MTP_MAGIC, MTP_VERSION, QUANT_AFFINE_INT4_G64, spec.num_layers, bb, h, I, V,
        spec.num_q_heads, spec.num_kv_heads, spec.head_dim, spec.global_head_dim, spec.global_kv_heads,
        spec.sliding_window, spec.global_layer_mask, GROUP, 1, offs[0][0], offs[0][1], offs[1][0], offs[1][1],
        offs[2][0], offs[2][1], offs[3][0], offs[3][1], *lo, *ls, hashlib.sha256(payload).digest(), b"\x00" * 3800)
    assert len(header) == HEADER_SIZE
    return header + payload


def write_mtp_container(path, spec: MtpSpec, seed: int = 0, centered: bool = False) -> Path:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_suffix(path.suffix + ".tmp")
    tmp.write_bytes(build_mtp_container(spec, seed, centered))
    tmp.replace(path)
    return path


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bf16 bit patterns (uint16)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    if not np.isfinite(x).all():
        u = u.astype(np.uint64)  # NaN/inf bit patterns could wrap in 32 bits
    rounded = (u + np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1))) >> 16
    return rounded.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def random_quant_block(rng: np.random.Generator, rows: int, cols: int, centered: bool = False):
    """Raw INT4 G64 block: (packed u32 [rows][cols/8], scales u16 [rows][cols/64],
    biases u16 [rows][cols/64]) with config-0 distributions.

    ``centered`` subtracts 7.5 * scale from each bias, making every group's dequantized
    weights zero-mean. BASELINE's distributions give the weights a large positive mean, which
    makes the greedy token stream nearly input-independent; the centered variant is a test
    aid that exercises input-dependent tokens with the same format and value ranges."""
    assert cols % GROUP == 0
    nib = rng.integers(0, 256, size=rows * cols // 2, dtype=np.uint8)
    packed = nib.view(np.uint32).reshape(rows, cols // 8)
    g = cols // GROUP
    s32 = np.abs(rng.standard_normal(rows * g, dtype=np.float32)) * 0.02
    scales = f32_to_bf16_bits(s32)
    b32 = rng.standard_normal(rows * g, dtype=np.float32) * 0.01
    if centered:
        b32 = b32 - 7.5 * bf16_bits_to_f32(scales)
    biases = f32_to_bf16_bits(b32)
    return packed, scales.reshape(rows, g), biases.reshape(rows, g)


def _norm(rng, n):
    return f32_to_bf16_bits(1.0 + rng.standard_normal(n, dtype=np.float32) * 0.05)


def _pad(buf: bytearray, align: int):
    rem = len(buf) % align
    if rem:
        buf += b"\x00" * (align - rem)


def _container_sections(spec: ModelSpec, seed: int, centered: bool):
    """Yields the payload in file order: the embedding block, then each layer block (each
    already padded to 4096 bytes), drawing from `default_rng(seed)` in the documented order."""
    rng = np.random.default_rng(seed)
    d, V = spec.d_model, spec.vocab_size

    def quant_bytes(rows, cols):
        p, s_, b_ = random_quant_block(rng, rows, cols, centered)
        return [p.tobytes(), s_.tobytes(), b_.tobytes()]

    def padded(parts, align):
        n = sum(len(x) for x in parts)
        return parts + [b"\x00" * ((-n) % align)]

    yield padded(quant_bytes(V, d) + [_norm(rng, d).tobytes()], ALIGNMENT)
    scalar = f32_to_bf16_bits(np.array([1.0 / np.sqrt(2.0 * spec.num_layers)], dtype=np.float32))
    for l in range(spec.num_layers):
        hd, _, _, _ = spec.layer_geometry(l)
        parts = [_norm(rng, d).tobytes() for _ in range(4)]
        parts += [_norm(rng, hd).tobytes(), _norm(rng, hd).tobytes(), scalar.tobytes()]
        for _, rows, cols in spec.layer_projections(l):
            n = sum(len(x) for x in parts)
            parts.append(b"\x00" * ((-n) % 16))
            parts += quant_bytes(rows, cols)
        yield padded(parts, ALIGNMENT)


def _header(spec: ModelSpec, embed_len: int, layer_lens, sha: bytes) -> bytes:
    offsets = [0] * 60
    sizes = [0] * 60
    cur = HEADER_SIZE + embed_len
    for l, n in enumerate(layer_lens):
        offsets[l], sizes[l] = cur, n
        cur += n
    layer_d_ff = [spec.d_ff] * spec.num_layers + [0] * (60 - spec.num_layers)
    header = struct.pack(
        HEADER_FMT, MAGIC, VERSION, QUANT_AFFINE_INT4_G64, spec.num_layers, spec.d_model, spec.d_ff,
        spec.num_q_heads, spec.num_kv_heads, spec.head_dim, spec.vocab_size, spec.sliding_window, GROUP,
        1, 1, spec.global_layer_mask, spec.rope_theta_local, spec.rope_theta_global, 1.0,
        spec.softcap, HEADER_SIZE, embed_len, HEADER_SIZE, embed_len, *offsets, *sizes, sha,
        spec.global_head_dim or (spec.head_dim if spec.global_layer_mask == 0 else 512),
        spec.global_kv_heads or (spec.num_kv_heads if spec.global_layer_mask == 0 else 4),
        0, 0, 0, 0, 0, 0, *layer_d_ff, 0, 0, 0.0, 0.0, b"\x00" * 2696)
    assert len(header) == HEADER_SIZE
    return header


def _write_sections(f, spec: ModelSpec, seed: int, centered: bool) -> bytes:
    """Writes header placeholder + payload to the open file `f`; returns the real header."""
    f.write(b"\x00" * HEADER_SIZE)
    sha = hashlib.sha256()
    lens = []
    for parts in _container_sections(spec, seed, centered):
        for x in parts:
            f.write(x)
            sha.update(x)
        lens.append(sum(len(x) for x in parts))
    return _header(spec, lens[0], lens[1:], sha.digest())


def build_container(spec: ModelSpec, seed: int = 0, centered: bool = False) -> bytes:
    """Returns the full container bytes for `spec` drawn from seed `seed` (see
    random_quant_block for ``centered``)."""
    import io
    buf = io.BytesIO()
    header = _write_sections(buf, spec, seed, centered)
    data = buf.getbuffer()
    data[:HEADER_SIZE] = header
    return bytes(data)


def write_container(path, spec: ModelSpec, seed: int = 0, centered: bool = False) -> Path:
    """Streams the container for `spec` to `path` (written to a temporary name, then renamed)."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_suffix(path.suffix + ".tmp")
    with open(tmp, "wb") as f:
        header = _write_sections(f, spec, seed, centered)
        f.seek(0)
        f.write(header)
    tmp.replace(path)
    return path


def layer_weight_ranges(spec: ModelSpec, l: int):
    """[(name, start, nbytes)] of each projection's packed nibble words inside layer l's block,
    following the writer's layout: six bf16 norms, the bf16 layer_scalar, then per projection a
    16-byte pad relative to the layer start and W, scales, biases."""
    hd, _, _, _ = spec.layer_geometry(l)
    off = 4 * spec.d_model * 2 + 2 * hd * 2 + 2
    out = []
    for name, rows, cols in spec.layer_projections(l):
        off += (-off) % 16
        w = rows * cols // 2
        out.append((name, off, w))
        off += w + 2 * (rows * cols // GROUP) * 2
    return out


def perturbed_copy(src, dst, spec: ModelSpec, frac: float, seed: int, embed_frac: float = 0.0) -> Path:
    """A test aid: a copy of container `src` (written for `spec`) in which a fraction `frac` of
    every layer projection's nibble bytes, and a fraction `embed_frac` of the tied embedding's
    nibble bytes, is re-drawn uniformly; norms, scales and biases stay as they are. Used as a
    drafter close to its target, so that speculative rounds accept some drafts and reject others.
    The header's payload sha256 is recomputed."""
    data = bytearray(Path(src).read_bytes())
    h = read_header(src)
    rng = np.random.default_rng(seed)

    def redraw(start, n, f):
        region = np.frombuffer(data, np.uint8, n, start).copy()
        hit = rng.random(n) < f
        region[hit] = rng.integers(0, 256, int(hit.sum()), dtype=np.uint8)
        data[start:start + n] = region.tobytes()

    if embed_frac > 0:
        redraw(h["embed_offset"], spec.vocab_size * spec.d_model // 2, embed_frac)
    for l in range(spec.num_layers):
        base = h["layer_offsets"][l]
        for _, start, n in layer_weight_ranges(spec, l):
            redraw(base + start, n, frac)
    sha_off = struct.calcsize("<IIIIIIIIIIIIIIQffffQQQQ60Q60Q")
    data[sha_off:sha_off + 32] = hashlib.sha256(bytes(data[HEADER_SIZE:])).digest()
    path = Path(dst)
    path.write_bytes(bytes(data))
    return path


def read_header(path) -> dict:
    with open(path, "rb") as f:
        raw = f.read(HEADER_SIZE)
    v = struct.unpack(HEADER_FMT, raw)
    keys = ["magic", "version", "quant_type", "num_layers", "d_model", "d_ff", "num_q_heads",
            "num_kv_heads", "head_dim", "vocab_size", "sliding_window", "quant_group_size",
            "scale_dtype", "tied_embeddings", "global_layer_mask", "rope_theta_local",
            "rope_theta_global", "rope_scaling", "final_logit_softcapping", "embed_offset",
            "embed_size", "lm_head_offset", "lm_head_size"]
    h = dict(zip(keys, v[:23]))
    h["layer_offsets"] = list(v[23:83])
    h["layer_sizes"] = list(v[83:143])
    h["global_head_dim"], h["global_kv_heads"] = v[144], v[145]
    return h


# ------------------------------------------- the reference's own test fixture (tiny.g4dense)

# Geometry of the fixture the reference's GPU tests run on (tools/make_synthetic_model.py:73-95,
# Gemma-4 variant): 4 sliding layers, d 256, FFN 512, 4 query heads over 2 KV heads of 64, a
# 1024-token vocabulary and a 512-key window.
REFERENCE_TINY = ModelSpec(num_layers=4, d_model=256, d_ff=512, num_q_heads=4, num_kv_heads=2, head_dim=64,
                           vocab_size=1024, sliding_window=512, global_head_dim=64, global_kv_heads=2)


def _bf16_truncated(x: np.ndarray) -> bytes:
    """float32 -> bf16 by dropping the low 16 bits (the fixture generator truncates; it does not
    round)."""
    return (np.ascontiguousarray(x, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16).tobytes()


def minmax_quant_g64(w: np.ndarray) -> bytes:
    """Affine INT4 G64 by each group's range, as the fixture generator quantizes real-valued
    weights (tools/make_synthetic_model.py:30-67): scale = (max - min) / 15 (1 where the range is
    0), bias = min, q = clip(round((w - min) / scale), 0, 15) with round-half-to-even, in float32.
    Returns the packed words, scales and biases in the container's order."""
    rows, cols = w.shape
    g = w.reshape(rows, cols // GROUP, GROUP)
    lo, hi = g.min(axis=-1, keepdims=True), g.max(axis=-1, keepdims=True)
    scale = (hi - lo) / np.float32(15.0)
    scale = np.where(scale == 0, np.float32(1.0), scale).astype(np.float32)
    q = np.clip(np.round((g - lo) / scale), 0, 15).astype(np.uint32).reshape(rows, cols)
    words = np.zeros((rows, cols // 8), dtype=np.uint32)
    for nib in range(8):
        words |= q[:, nib::8] << np.uint32(4 * nib)
    return words.tobytes() + _bf16_truncated(scale) + _bf16_truncated(lo)


def reference_tiny_container(seed: int = 42) -> bytes:
    """The reference's tests/fixtures/tiny.g4dense, byte for byte (its generator,
    tools/make_synthetic_model.py, with the default seed 42 and the Gemma-4 architecture).

    Weights are N(0, 0.02) from the legacy global NumPy generator seeded with `seed`, drawn in
    this order: the embedding [V][d]; then per layer q, k, v, o, gate, up, down. Each is quantized
    by minmax_quant_g64. Every norm weight is 1, layer_scalar is 1/sqrt(2L), and both are bf16 by
    truncation. Blocks follow the container layout and are padded to 4096 bytes. The header also
    records attn_out_dim = d, qk_scale_factor = output_multiplier = 1 and the per-layer FFN widths."""
    spec = REFERENCE_TINY
    rng = np.random.RandomState(seed)
    d, f, V, L = spec.d_model, spec.d_ff, spec.vocab_size, spec.num_layers
    qd, kvd = spec.num_q_heads * spec.head_dim, spec.num_kv_heads * spec.head_dim

    def gauss(rows, cols):
        return (rng.randn(rows, cols).astype(np.float32) * np.float32(0.02)).astype(np.float32)

    ones = lambda n: _bf16_truncated(np.ones(n, dtype=np.float32))  # noqa: E731
    embed = bytearray(minmax_quant_g64(gauss(V, d)) + ones(d))
    _pad(embed, ALIGNMENT)
    scalar = _bf16_truncated(np.array([1.0 / np.sqrt(2.0 * L)], dtype=np.float32))
    layers = []
    for _ in range(L):
        mats = [gauss(qd, d), gauss(kvd, d), gauss(kvd, d), gauss(d, qd), gauss(f, d), gauss(f, d), gauss(d, f)]
        # the four [d] norms, q_norm and k_norm [head_dim], layer_scalar
        block = bytearray(ones(d) + ones(d) + ones(d) + ones(d) + ones(spec.head_dim) + ones(spec.head_dim) + scalar)
        for m in mats:
            _pad(block, 16)
            block += minmax_quant_g64(m)
        _pad(block, ALIGNMENT)
        layers.append(bytes(block))
    payload = bytes(embed) + b"".join(layers)
    offsets, sizes, cur = [0] * 60, [0] * 60, HEADER_SIZE + len(embed)
    for l, b in enumerate(layers):
        offsets[l], sizes[l] = cur, len(b)
        cur += len(b)
    header = struct.pack(
        HEADER_FMT, MAGIC, VERSION, QUANT_AFFINE_INT4_G64, L, d, f, spec.num_q_heads, spec.num_kv_heads,
        spec.head_dim, V, spec.sliding_window, GROUP, 1, 1, 0, spec.rope_theta_local, spec.rope_theta_global, 1.0,
        spec.softcap, HEADER_SIZE, len(embed), HEADER_SIZE, len(embed), *offsets, *sizes,
        hashlib.sha256(payload).digest(), spec.global_head_dim, spec.global_kv_heads, 0, 0, 0, 0, 0, 0,
        *([f] * L + [0] * (60 - L)), 0, d, 1.0, 1.0, b"\x00" * 2696)
    return header + payload
