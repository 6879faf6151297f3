"""The container verifier g4dense_b200.verify (CPU only): every container the converters and the
synthetic writers make passes; a flipped payload byte, a wrong magic word or version, a misaligned,
empty or out-of-file block and a short header are each reported."""
from __future__ import annotations

import struct

import pytest

from g4dense_b200 import container as C
from g4dense_b200 import convert as V
from g4dense_b200 import synth_checkpoint as S
from g4dense_b200 import verify as W


@pytest.mark.parametrize("kind, name", [("model", n) for n, c in S.converter_cases().items() if c[4]] +
                         [("assistant", n) for n, c in S.assistant_cases().items() if c[4]])
def test_converted_containers_verify(kind, name, tmp_path):
    cases = S.converter_cases() if kind == "model" else S.assistant_cases()
    config, tensors, prefix, shards, _ = cases[name]
    ck = S.write_checkpoint(tmp_path / "ck", config, tensors, prefix, shards)
    out = (V.convert if kind == "model" else V.convert_assistant)(ck, tmp_path / "c.out")
    info = W.verify_container(out)
    assert info["kind"] == ("g4dense" if kind == "model" else "g4mtp")
    assert info["size"] == out.stat().st_size


def _model(tmp_path):
    return C.write_container(tmp_path / "m.g4dense", C.CONFIG0_TARGET, 0)


def _assistant(tmp_path):
    return C.write_mtp_container(tmp_path / "a.g4mtp", C.MtpSpec.for_target(C.MTP_TEST_TARGET), 0)


def test_synthetic_containers_verify(tmp_path, capsys):
    m, a = _model(tmp_path), _assistant(tmp_path)
    assert W.verify_container(m)["layers"] == C.CONFIG0_TARGET.num_layers
    assert W.verify_container(a)["backbone"] == C.MTP_TEST_TARGET.d_model
    assert W.main([str(m), str(a)]) == 0
    assert capsys.readouterr().out.count("OK ") == 2


def _patch(path, offset, data: bytes):
    raw = bytearray(path.read_bytes())
    raw[offset:offset + len(data)] = data
    path.write_bytes(bytes(raw))


# Byte offsets inside the .g4dense header: the version at 4, then the layer offsets and layer sizes
# tables (60 u64 each) after the geometry fields and the four block offset/size words.
_LAYER_OFFSETS = struct.calcsize("<IIIIIIIIIIIIIIQffffQQQQ")
_LAYER_SIZES = _LAYER_OFFSETS + 60 * 8


@pytest.mark.parametrize("damage, message", [
    (lambda p: _patch(p, C.HEADER_SIZE + 1000, bytes([p.read_bytes()[C.HEADER_SIZE + 1000] ^ 1])), "SHA-256"),
    (lambda p: _patch(p, 0, struct.pack("<I", 0x12345678)), "magic word"),
    (lambda p: _patch(p, 4, struct.pack("<I", 2)), "format version 2"),
    (lambda p: _patch(p, _LAYER_OFFSETS + 8, struct.pack("<Q", struct.unpack_from(
        "<Q", p.read_bytes(), _LAYER_OFFSETS + 8)[0] + 16)), "layer 1 starts"),
    (lambda p: _patch(p, _LAYER_SIZES + 8 * 2, struct.pack("<Q", 0)), "layer 2 is empty"),
    (lambda p: p.write_bytes(p.read_bytes()[:-4096]), "outside the"),
    (lambda p: p.write_bytes(p.read_bytes()[:100]), "shorter than"),
], ids=["payload", "magic", "version", "misaligned", "empty", "truncated", "short_header"])
def test_damage_is_reported(damage, message, tmp_path, capsys):
    p = _model(tmp_path)
    damage(p)
    with pytest.raises(W.ContainerError, match=message):
        W.verify_container(p)
    assert W.main([str(p)]) == 1
    assert message.split()[0] in capsys.readouterr().err


def test_assistant_damage_is_reported(tmp_path):
    a = _assistant(tmp_path)
    raw = bytearray(a.read_bytes())
    raw[-1] ^= 0xFF
    a.write_bytes(bytes(raw))
    with pytest.raises(W.ContainerError, match="SHA-256"):
        W.verify_container(a)
    b = _assistant(tmp_path)
    _patch(b, 4, struct.pack("<I", 3))
    with pytest.raises(W.ContainerError, match="g4mtp format version 3"):
        W.verify_container(b)


def test_per_layer_input_block_is_checked(tmp_path):
    """A container with per-layer inputs (E2B-style) verifies, and its per-layer-input block is one
    of the blocks checked: moved off its page, it is reported."""
    config, tensors, prompt = S.forward_cases()["e2b_ple_shared_kv"]
    ck = S.write_checkpoint(tmp_path / "ck", config, tensors, prefix="model.")
    out = V.convert(ck, tmp_path / "e2b.g4dense")
    assert W.verify_container(out)["kind"] == "g4dense"
    ple_offset = struct.calcsize("<IIIIIIIIIIIIIIQffffQQQQ60Q60Q32sIIIIII")
    _patch(out, ple_offset, struct.pack("<Q", struct.unpack_from("<Q", out.read_bytes(), ple_offset)[0] + 8))
    with pytest.raises(W.ContainerError, match="per-layer-input block starts"):
        W.verify_container(out)
