"""Header validation of the engine's loader, through g4dense_container_validate (CPU only; the
check reads the header and the file size and touches no GPU).

The cases follow the reference's tests/test_format.cpp: a valid model and assistant header are
accepted; a bad magic word, a block off its 4096-byte page and a file too short for its blocks
are rejected. Added: the layer-count bounds, the format version, and what this engine refuses to
run with the reason (Muse-Glimmer, per-layer embeddings, an untied head, another quantization, a
width that is not whole 64-groups, a head_dim the kernels lack, a layer block shorter than its
tensors). Several broken rules are reported together.
"""
from __future__ import annotations

import struct

import pytest

from g4dense_b200 import api
from g4dense_b200 import container as C
from g4dense_b200 import convert as V
from g4dense_b200 import synth_checkpoint as S

# Field indices of struct.unpack(C.HEADER_FMT) and struct.unpack(C.MTP_HEADER_FMT).
MAGIC, VERSION, QUANT, LAYERS, D_MODEL, D_FF = 0, 1, 2, 3, 4, 5
GROUP, TIED, EMBED_OFF, LM_OFF, LAYER_OFF, LAYER_SIZE = 11, 13, 19, 21, 23, 83
PLE_DIM, LAYER_D_FF, ARCH = 146, 152, 212
M_LAYERS, M_HIDDEN, M_PRE_OFF, M_LAYER_OFF = 3, 5, 19, 25


def _edit(path, fmt, **changes):
    raw = bytearray(path.read_bytes())
    fields = list(struct.unpack(fmt, bytes(raw[:C.HEADER_SIZE])))
    for index, value in changes.items():
        fields[int(index[1:])] = value
    raw[:C.HEADER_SIZE] = struct.pack(fmt, *fields)
    path.write_bytes(bytes(raw))
    return path


def _model(tmp_path, name="m.g4dense", spec=C.CONFIG0_TARGET):
    return C.write_container(tmp_path / name, spec, 0)


def _assistant(tmp_path):
    return C.write_mtp_container(tmp_path / "a.g4mtp", C.MtpSpec.for_target(C.MTP_TEST_TARGET), 0)


def _rejects(path, *phrases):
    with pytest.raises(ValueError) as e:
        api.validate_container(path)
    for p in phrases:
        assert p in str(e.value), str(e.value)
    return str(e.value)


def test_valid_containers(tmp_path):
    assert api.validate_container(_model(tmp_path)) == "g4dense"
    assert api.validate_container(_model(tmp_path, "g.g4dense", C.MTP_TEST_TARGET)) == "g4dense"
    assert api.validate_container(_assistant(tmp_path)) == "g4mtp"


def test_converted_container_is_accepted(tmp_path):
    spec = C.CONFIG0_TARGET
    ck = S.write_checkpoint(tmp_path / "ck", S.gemma4_config(spec), S.gemma4_tensors(spec, 0))
    assert api.validate_container(V.convert(ck, tmp_path / "c.g4dense")) == "g4dense"


@pytest.mark.parametrize("case, phrase", [
    ("untied_head", "tied embedding"),
    ("ple_shared_kv", "per-layer embeddings"),
    ("muse_glimmer_defaults", "architecture 1"),
])
def test_engine_refuses_other_architectures(case, phrase, tmp_path):
    config, tensors, prefix, shards, _ = S.converter_cases()[case]
    ck = S.write_checkpoint(tmp_path / "ck", config, tensors, prefix, shards)
    _rejects(V.convert(ck, tmp_path / "c.g4dense"), phrase)


F = C.HEADER_FMT


@pytest.mark.parametrize("changes, phrases", [
    ({"f0": 0xDEADBEEF}, ["magic word is 0xDEADBEEF"]),
    ({"f1": 2}, ["format version 2"]),
    ({f"f{LAYER_OFF}": 4097}, ["layer 0 starts at byte 4097"]),
    ({f"f{EMBED_OFF}": 4096 + 512}, ["embedding block starts at byte 4608"]),
    ({f"f{LAYERS}": 0}, ["0 layers"]),
    ({f"f{LAYERS}": 61}, ["61 layers"]),
    ({f"f{LAYER_SIZE + 2}": 0}, ["layer 2 is empty"]),
    ({f"f{QUANT}": 2}, ["quantization 2"]),
    ({f"f{GROUP}": 32}, ["group 32"]),
    ({f"f{D_MODEL}": 0}, ["zero-sized geometry"]),
    ({f"f{D_MODEL}": 200}, ["d_model 200"]),
    ({f"f{TIED}": 0}, ["tied embedding"]),
    ({f"f{LM_OFF}": 8192}, ["tied embedding"]),
    ({f"f{ARCH}": 1}, ["architecture 1"]),
    ({f"f{PLE_DIM}": 256}, ["per-layer embeddings"]),
    ({f"f{QUANT}": 2, f"f{ARCH}": 1}, ["(2 problems)", "quantization 2", "architecture 1"]),
    ({f"f{LAYER_SIZE + 1}": 4096}, ["layer 1 holds 4096 bytes; its tensors need"]),
    ({"f8": 96}, ["head_dim 96"]),
    ({f"f{LAYER_D_FF}": 1000}, ["layer 0: FFN width 1000"]),  # the per-layer width the engine uses
], ids=["magic", "version", "layer_misaligned", "embed_misaligned", "no_layers", "61_layers", "empty_layer",
        "quant_type", "group", "zero_width", "width_not_64", "untied", "lm_head_elsewhere", "muse", "ple",
        "two_problems", "layer_too_short", "head_dim", "ffn_width"])
def test_model_header_rejections(changes, phrases, tmp_path):
    _rejects(_edit(_model(tmp_path), F, **changes), *phrases)


def test_file_bounds(tmp_path):
    p = _model(tmp_path)
    raw = p.read_bytes()
    p.write_bytes(raw[:-100])
    _rejects(p, "past the end")
    p.write_bytes(raw[:4000])
    _rejects(p, "too small for header")
    # A layer whose end wraps around 64 bits.
    q = _edit(_model(tmp_path, "w.g4dense"), F, **{f"f{LAYER_SIZE}": 2**64 - 4096})
    _rejects(q, "overflows 64 bits")
    _rejects(tmp_path / "absent.g4dense", "cannot open")


M = C.MTP_HEADER_FMT


@pytest.mark.parametrize("changes, phrases", [
    ({"f1": 2}, ["format version 2"]),
    ({f"f{M_LAYERS}": 9}, ["9 layers"]),
    ({f"f{M_HIDDEN}": 0}, ["zero-sized geometry"]),
    ({f"f{M_HIDDEN}": 100}, ["whole numbers of 64-wide groups"]),
    ({f"f{M_PRE_OFF}": 4100}, ["pre-projection section starts at byte 4100"]),
    ({f"f{M_LAYER_OFF + 1}": 10**12}, ["drafter layer 1", "past the end"]),
    ({f"f{QUANT}": 3}, ["quantization 3"]),
], ids=["version", "nine_layers", "zero_hidden", "hidden_not_64", "pre_misaligned", "layer_outside", "quant"])
def test_assistant_header_rejections(changes, phrases, tmp_path):
    _rejects(_edit(_assistant(tmp_path), M, **changes), *phrases)
