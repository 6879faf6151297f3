"""The checkpoint converters g4dense_b200.convert.convert (.g4dense) and convert_assistant
(.g4mtp) (CPU only).

1. Against the reference converters: every synthetic checkpoint of converter_cases() and
   assistant_cases() converts to the same container, byte for byte, as
   tools/convert_hf_to_g4dense.py or tools/convert_hf_assistant.py wrote for it
   (tests/golden/convert.json, made by tests/golden/make_convert_golden.py), and the checkpoints
   the reference refuses are refused.
2. Against the synthetic container writers: a Gemma-4 checkpoint drawn as
   container.build_container draws converts to that container's payload, and to its header up to
   the three fields the synthetic writer leaves zero; an assistant checkpoint drawn as
   build_mtp_container draws converts to that container, header included.
3. The converted container loads in the CPU oracle and gives the same logits as the synthetic one.
"""
from __future__ import annotations

import dataclasses
import hashlib
import json
import struct
from pathlib import Path

import numpy as np
import pytest

from g4dense_b200 import container as C
from g4dense_b200 import convert as V
from g4dense_b200 import synth_checkpoint as S

GOLDEN = json.loads((Path(__file__).parent / "golden" / "convert.json").read_text())
CASES = {"model": S.converter_cases(), "assistant": S.assistant_cases()}
CONVERTERS = {"model": V.convert, "assistant": V.convert_assistant}


def test_golden_covers_every_case():
    assert {k: sorted(v) for k, v in GOLDEN.items()} == {k: sorted(v) for k, v in CASES.items()}


@pytest.mark.parametrize("kind, name", [(k, n) for k in sorted(CASES) for n in sorted(CASES[k])])
def test_matches_reference_converter(kind, name, tmp_path):
    config, tensors, prefix, shards, converts = CASES[kind][name]
    want = GOLDEN[kind][name]
    assert S.tensors_digest(tensors) == want["tensors"], \
        "the synthetic checkpoint changed: regenerate tests/golden/convert.json"
    ck = S.write_checkpoint(tmp_path / "ck", config, tensors, prefix, shards)
    out = tmp_path / "m.out"
    if not converts:
        assert want.get("refused")
        with pytest.raises(V.CheckpointError):
            CONVERTERS[kind](ck, out)
        assert not out.exists() and not (tmp_path / "m.out.tmp").exists()
        return
    data = CONVERTERS[kind](ck, out).read_bytes()
    assert len(data) == want["size"]
    assert hashlib.sha256(data).hexdigest() == want["sha256"]
    assert not (tmp_path / "m.out.tmp").exists()


@pytest.mark.parametrize("layers", [1, 4, 8])
def test_assistant_equals_synthetic_container(layers, tmp_path):
    spec = C.MtpSpec.for_target(C.MTP_TEST_TARGET, num_layers=layers)
    ck = S.write_checkpoint(tmp_path / "ck", S.assistant_config(spec), S.assistant_tensors(spec, 9, centered=True),
                            prefix="", shards=2)
    got = V.convert_assistant(ck, tmp_path / "a.g4mtp").read_bytes()
    assert got == C.build_mtp_container(spec, 9, centered=True)


def test_assistant_geometry():
    g = V.assistant_geometry({})
    assert (g["num_hidden_layers"], g["backbone"], g["hidden_size"], g["intermediate_size"], g["vocab_size"]) == \
        (4, 5376, 1024, 8192, 262144)
    assert (g["num_key_value_heads"], g["head_dim"], g["global_head_dim"], g["num_global_key_value_heads"]) == \
        (16, 256, 512, 4)
    assert g["mask"] == 0b1000
    g = V.assistant_geometry({"backbone_hidden_size": 256, "text_config": {
        "num_hidden_layers": 2, "layer_types": ["full_attention", "sliding_attention"]}})
    assert (g["backbone"], g["mask"]) == (256, 0b01)
    for L in (0, 9):
        with pytest.raises(V.CheckpointError, match="1..8"):
            V.assistant_geometry({"num_hidden_layers": L})


_HEADER_FIELDS_ZERO_IN_SYNTH = ("attn_out_dim", "qk_scale_factor", "output_multiplier")


def _fields(raw: bytes) -> list:
    return list(struct.unpack(C.HEADER_FMT, raw[:C.HEADER_SIZE]))


@pytest.mark.parametrize("spec", [C.CONFIG0_TARGET, C.CONFIG0_DRAFT, C.MID_TEST_DRAFT,
                                  dataclasses.replace(C.CONFIG0_TARGET, global_layer_mask=0b0110,
                                                      global_head_dim=128, global_kv_heads=2)],
                         ids=["config0_target", "config0_draft", "mid_draft", "global_layers"])
def test_payload_equals_synthetic_container(spec, tmp_path):
    ck = S.write_checkpoint(tmp_path / "ck", S.gemma4_config(spec), S.gemma4_tensors(spec, 7, centered=True),
                            shards=2)
    got = V.convert(ck, tmp_path / "m.g4dense").read_bytes()
    want = C.build_container(spec, 7, centered=True)
    assert got[C.HEADER_SIZE:] == want[C.HEADER_SIZE:]
    g, w = _fields(got), _fields(want)
    # The header's tail: ..., layer_d_ff[60], arch_type, attn_out_dim, qk_scale_factor,
    # output_multiplier, reserved. The synthetic writer leaves the middle three zero.
    assert g[:-4] == w[:-4] and g[-1] == w[-1]
    assert w[-4:-1] == [0, 0.0, 0.0]
    assert g[-4:-1] == [spec.d_model, 1.0, 1.0]
    h = C.read_header(tmp_path / "m.g4dense")
    assert h["tied_embeddings"] == 1 and h["lm_head_offset"] == h["embed_offset"] == C.HEADER_SIZE
    assert h["global_layer_mask"] == spec.global_layer_mask


def test_converted_container_runs_in_oracle(tmp_path):
    from oracle import oracle as O
    spec = C.CONFIG0_TARGET
    ck = S.write_checkpoint(tmp_path / "ck", S.gemma4_config(spec), S.gemma4_tensors(spec, 0, centered=True))
    conv = V.convert(ck, tmp_path / "conv.g4dense")
    synth = C.write_container(tmp_path / "synth.g4dense", spec, 0, centered=True)
    a, b = O.RestatedModel(str(conv)), O.RestatedModel(str(synth))
    try:
        for pos, tok in enumerate([2, 105, 17, 900, 4095, 3]):
            la, lb = a.forward(tok, pos), b.forward(tok, pos)
            assert np.array_equal(la, lb)
    finally:
        a.close()
        b.close()


def test_geometry_defaults_follow_architecture():
    g = V.geometry({"text_config": {"layer_types": ["sliding_attention"] * 60}})
    assert (g["layers"], g["d_model"], g["d_ff"], g["kv_heads"], g["head_dim"], g["vocab"]) == \
        (60, 5376, 21504, 16, 256, 262144)
    assert (g["window"], g["softcap"], g["global_head_dim"], g["global_kv_heads"]) == (1024, 30.0, 512, 16)
    assert (g["theta_local"], g["theta_global"], g["tied"], g["attn_out_dim"]) == (10000.0, 1000000.0, True, 5376)
    m = V.geometry({"model_type": "muse_glimmer", "text_config": {"layer_types": ["full_attention"] * 52}})
    assert m["muse"] and not m["tied"]
    assert (m["layers"], m["d_model"], m["kv_heads"], m["head_dim"], m["vocab"], m["window"]) == \
        (52, 6656, 2, 128, 202048, 2048)
    assert (m["attn_out_dim"], m["global_head_dim"], m["qk_scale"], m["theta_global"]) == (4096, 128, 3.87, 0.0)
    assert m["mask"] == (1 << 52) - 1


@pytest.mark.parametrize("text_config, message", [
    ({"num_experts": 4, "layer_types": ["sliding_attention"]}, "mixture-of-experts"),
    ({"num_hidden_layers": 2}, "layer_types"),
    ({"num_hidden_layers": 61, "layer_types": ["sliding_attention"] * 61}, "at most 60"),
    ({"num_hidden_layers": 4, "layer_types": ["sliding_attention"] * 3}, "layer_types"),
])
def test_geometry_refusals(text_config, message):
    with pytest.raises(V.CheckpointError, match=message):
        V.geometry({"text_config": text_config})


def test_cli_reports_errors(tmp_path, capsys):
    assert V.main(["--input", str(tmp_path), "--out", str(tmp_path / "x.g4dense")]) == 1
    assert "no config.json" in capsys.readouterr().err
    spec = C.CONFIG0_DRAFT
    ck = S.write_checkpoint(tmp_path / "ck", S.gemma4_config(spec), S.gemma4_tensors(spec, 0))
    t = S.gemma4_tensors(spec, 0)
    del t["layers.1.mlp.up_proj.weight"]
    bad = S.write_checkpoint(tmp_path / "bad", S.gemma4_config(spec), t)
    assert V.main(["--input", str(bad), "--out", str(tmp_path / "bad.g4dense")]) == 1
    assert "layers.1.mlp.up_proj.weight" in capsys.readouterr().err
    assert not (tmp_path / "bad.g4dense").exists() and not (tmp_path / "bad.g4dense.tmp").exists()
    assert V.main(["--input", str(ck), "--out", str(tmp_path / "ok.g4dense")]) == 0
    assert (tmp_path / "ok.g4dense").read_bytes() == V.convert(ck, tmp_path / "again.g4dense").read_bytes()
    mspec = C.MtpSpec.for_target(C.MTP_TEST_TARGET)
    ack = S.write_checkpoint(tmp_path / "ack", S.assistant_config(mspec), S.assistant_tensors(mspec, 0), prefix="")
    assert V.main(["--assistant", "--input-dir", str(ack), "--output-file", str(tmp_path / "a.g4mtp")]) == 0
    assert (tmp_path / "a.g4mtp").read_bytes() == C.build_mtp_container(mspec, 0)


def test_small_chunks_give_the_same_container(tmp_path, monkeypatch):
    """Tensors are copied in bounded chunks; a chunk far smaller than every tensor (so each is
    copied in many pieces, ragged last piece included) writes the same bytes."""
    config, tensors, prefix, shards, _ = CASES["model"]["global_layers_bare_names"]
    ck = S.write_checkpoint(tmp_path / "ck", config, tensors, prefix, shards)
    whole = V.convert(ck, tmp_path / "whole.g4dense").read_bytes()
    monkeypatch.setattr(V._Span, "CHUNK", 1000)
    assert V.convert(ck, tmp_path / "chunked.g4dense").read_bytes() == whole
    assert hashlib.sha256(whole).hexdigest() == GOLDEN["model"]["global_layers_bare_names"]["sha256"]


def test_shard_shorter_than_its_index_is_refused(tmp_path):
    spec = C.CONFIG0_DRAFT
    ck = S.write_checkpoint(tmp_path / "ck", S.gemma4_config(spec), S.gemma4_tensors(spec, 0))
    shard = next(ck.glob("*.safetensors"))
    shard.write_bytes(shard.read_bytes()[:-10])
    with pytest.raises(V.CheckpointError, match="outside shard"):
        V.convert(ck, tmp_path / "m.g4dense")
    assert not (tmp_path / "m.g4dense").exists()
