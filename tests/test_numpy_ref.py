"""Checkpoint -> converter -> oracle against the reference's independent NumPy forward pass
(CPU only).

tests/golden/numpy_ref.json holds the logits that the reference's tools/numpy_reference.py
computes straight from each synthetic MLX checkpoint of forward_cases() (made by
tests/golden/make_numpy_ref_golden.py). Here the same checkpoint goes through this library's
converter, and the oracle (the restatement of the reference's CPU runner) runs the container. The
two must agree position by position within BASELINE's logits tolerance, 2e-2 of the row's max
|logit|, with the same argmax and top-5 order wherever the reference's gaps leave room for the
fp16 KV rounding of the CPU runner (0.05 between neighbours). This pins what the converter's
bytes mean, not only the bytes, and checks the oracle against a second implementation of the
reference that shares no code with the first (global layers, partial rotary, GQA, window wrap).
The E2B-style cases (per-layer inputs, layers reading another layer's K/V, a double-wide FFN)
check the oracle's restatement of that path of the reference's GPU runner, for which the
reference has no C++ CPU code: the NumPy pass is the reference's only CPU implementation of it.
"""
from __future__ import annotations

import base64
import json
from pathlib import Path

import numpy as np
import pytest

from g4dense_b200 import convert as V
from g4dense_b200 import synth_checkpoint as S
from oracle import oracle as O

GOLDEN = json.loads((Path(__file__).parent / "golden" / "numpy_ref.json").read_text())
CASES = S.forward_cases()
TOL = 2e-2     # BASELINE: logits within 2e-2 of the row's max |logit|
MARGIN = 0.05  # order checks only where neighbouring reference logits are this far apart
# With an fp32 K/V cache, as the NumPy pass keeps it, what remains is summation order and the
# fixture's fp16 storage of the logits (at most max|z| * 2^-11, about 5e-4 of the row's max).
TOL_FP32_KV = 2e-3


def _reference_rows(name):
    return [np.frombuffer(base64.b64decode(b), dtype="<f2").astype(np.float32)
            for b in GOLDEN[name]["logits_f16"]]


def _e2b(config) -> bool:
    return bool(config["text_config"].get("hidden_size_per_layer_input"))


def _oracle_rows(tmp_path, config, tensors, prompt, kv_mode=O.KV_FP16):
    ck = S.write_checkpoint(tmp_path / "ck", config, tensors, prefix="model.")
    m = O.RestatedModel(str(V.convert(ck, tmp_path / "m.g4dense")), kv_mode=kv_mode)
    try:
        return [np.asarray(m.forward(t, p), dtype=np.float32).copy() for p, t in enumerate(prompt)]
    finally:
        m.close()


def test_golden_covers_every_case():
    assert sorted(GOLDEN) == sorted(CASES)


@pytest.mark.parametrize("name", sorted(CASES))
def test_converted_checkpoint_matches_numpy_reference(name, tmp_path):
    config, tensors, prompt = CASES[name]
    assert S.tensors_digest(tensors) == GOLDEN[name]["tensors"], \
        "the synthetic checkpoint changed: regenerate tests/golden/numpy_ref.json"
    assert GOLDEN[name]["prompt"] == prompt
    ordered = 0
    for p, (ours, ref) in enumerate(zip(_oracle_rows(tmp_path, config, tensors, prompt), _reference_rows(name))):
        rel = np.abs(ours - ref).max() / np.abs(ref).max()
        assert rel <= TOL, f"position {p}: max |diff| is {rel:.2e} of the row's max"
        top = np.argsort(-ref, kind="stable")[:6]
        gaps = -np.diff(ref[top])
        # Compare the top-5 order up to the first near-tie, as the reference's GPU-vs-CPU test does.
        k = next((i for i, g in enumerate(gaps[:5]) if g < MARGIN), 5)
        assert list(np.argsort(-ours, kind="stable")[:k]) == list(top[:k]), f"position {p}: top-{k} order"
        ordered += k > 0
    assert ordered >= len(prompt) - 1  # at most one position too close to call
    # The same arithmetic with the cache kept in fp32: the two implementations agree to the
    # fixture's storage precision.
    for p, (ours, ref) in enumerate(zip(_oracle_rows(tmp_path / "f32", config, tensors, prompt, O.KV_FP32),
                                        _reference_rows(name))):
        rel = np.abs(ours - ref).max() / np.abs(ref).max()
        assert rel <= TOL_FP32_KV, f"position {p} (fp32 K/V): max |diff| is {rel:.2e} of the row's max"


def test_fixture_catches_a_window_off_by_one(tmp_path):
    """A mistake planted in the input (the converted config's window one key short) must fail the
    tolerance: the fixture is sensitive to the sliding-window semantics."""
    config, tensors, prompt = CASES["window_wrap"]
    bad = json.loads(json.dumps(config))
    bad["text_config"]["sliding_window"] -= 1
    worst = max(np.abs(o - r).max() / np.abs(r).max()
                for o, r in zip(_oracle_rows(tmp_path, bad, tensors, prompt), _reference_rows("window_wrap")))
    assert worst > 10 * TOL


def test_fixture_catches_a_missing_per_layer_input_block(tmp_path):
    """The same for the per-layer-input path: with every layer's per_layer_projection silenced
    (zero scales and biases) in the converted input, the E2B case falls far outside tolerance."""
    config, tensors, prompt = CASES["e2b_ple_shared_kv_global"]
    bad = dict(tensors)
    for name, (dtype, shape, data) in tensors.items():
        if name.endswith("per_layer_projection.scales") or name.endswith("per_layer_projection.biases"):
            bad[name] = (dtype, shape, bytes(len(data)))
    worst = max(np.abs(o - r).max() / np.abs(r).max()
                for o, r in zip(_oracle_rows(tmp_path, config, bad, prompt), _reference_rows("e2b_ple_shared_kv_global")))
    assert worst > 5 * TOL


@pytest.mark.skipif(not O.reference_available(), reason="oracle/_ref (the reference's compiled CPU runner) not built")
@pytest.mark.parametrize("name", sorted(n for n, c in CASES.items() if not _e2b(c[0])))
def test_oracle_equals_reference_cpu_runner_on_converted_containers(name, tmp_path):
    """On the same converted containers the oracle equals the reference's own compiled CPU runner
    bit for bit, so the gap to the NumPy pass (up to 1.55e-2 of the row's max on the wrapping
    window) lies between the reference's two implementations: the CPU runner's fp16 K/V cache
    against the NumPy pass's fp32 one."""
    config, tensors, prompt = CASES[name]
    ck = S.write_checkpoint(tmp_path / "ck", config, tensors, prefix="model.")
    path = str(V.convert(ck, tmp_path / "m.g4dense"))
    m, r = O.RestatedModel(path), O.ReferenceModel(path)
    try:
        for p, t in enumerate(prompt):
            assert np.array_equal(np.asarray(m.forward(t, p), dtype=np.float32),
                                  np.asarray(r.forward(t, p), dtype=np.float32)), f"position {p}"
    finally:
        m.close()
        r.close()
