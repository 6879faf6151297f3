"""Pins the CPU oracle before anything is checked against it (CPU only).

1. Known answers copied from the reference's own tests: splitmix64 constants
   (tests/test_sampling.cpp:118-121), greedy acceptance cases (tests/test_speculative.cpp:29-77),
   greedy tie to the lowest index (tests/test_sampling.cpp:139-149), validate_sampling's
   rejection table (tests/test_sampling.cpp:92-112).
2. Golden vectors produced by the reference's CPU code (tests/golden/config0.json, made by
   tests/golden/make_golden.py): the restated forward pass must reproduce the reference's
   logits bit for bit, and the restated decode loop its token streams and per-round decisions.
3. When oracle/_ref is built, a live cross-check against it (including the sampled path's
   mt19937_64 draws).
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = json.loads((Path(__file__).parent / "golden" / "config0.json").read_text())


def test_splitmix64_known_answers():
    lib = O.restated_lib()
    expected = {0: 0xE220A8397B1DCDAF, 1: 0x910A2DEC89025CC1, 2: 0x975835DE1C9756CE, 3: 0x1D0B14E4DB018FED}
    for x, v in expected.items():
        assert lib.g4o_splitmix64(x) == v
        assert int(GOLDEN["splitmix64"][str(x)], 16) == v


def test_seed_for_never_zero_and_stable():
    lib = O.restated_lib()
    sp = O.Sampling(0.7, 1.0, 0, 1.0, 1, 12345)
    seeds = [lib.g4o_seed_for(sp, p) for p in range(2000)]
    assert all(s != 0 for s in seeds)
    assert seeds == [lib.g4o_seed_for(sp, p) for p in range(2000)]
    assert seeds[0] != seeds[1]


def _onehot_targets():
    t = np.zeros((5, 1024), np.float32)
    for i, a in enumerate([42, 100, 200, 300, 400]):
        t[i, a] = 10.0
    return t


def test_greedy_acceptance_known_answers():
    t = _onehot_targets()
    assert O.evaluate_verification([42, 100, 200, 300], t, base_seed=12345) == ([42, 100, 200, 300, 400], 4)
    assert O.evaluate_verification([42, 100, 999, 300], t, base_seed=12345) == ([42, 100, 200], 2)
    assert O.evaluate_verification([999, 100], t, base_seed=12345) == ([42], 0)


def test_greedy_tie_lowest_index():
    lib = O.restated_lib()
    logits = np.array([1.0, 5.0, 3.0, 5.0, 2.0], np.float32)
    sp = O.Sampling.greedy()
    assert lib.g4o_sample_token(logits.ctypes.data, 5, sp, 1) == 1
    one = np.array([7.0], np.float32)
    assert lib.g4o_sample_token(one.ctypes.data, 1, sp, 1) == 0


@pytest.mark.parametrize("params,rejected", [
    ((0.2, 0.95, 64, 1.0), False), ((0.0, 1.0, 0, 1.0), False), ((-0.1, 1.0, 0, 1.0), True),
    ((0.2, 0.0, 64, 1.0), True), ((0.2, 1.5, 64, 1.0), True), ((0.2, 0.95, 257, 1.0), True),
    ((0.2, 0.95, -1, 1.0), True), ((0.2, 0.95, 64, 0.0), True), ((0.7, 0.9, 0, 1.0), True),
    ((0.7, 1.0, 0, 1.0), False), ((0.0, 0.9, 0, 1.0), False)])
def test_validate_sampling_table(params, rejected):
    lib = O.restated_lib()
    t, p, k, r = params
    assert (lib.g4o_validate_sampling(O.Sampling(t, p, k, r, 0, 0)) != 0) == rejected


def test_fp16_round_trip_matches_reference_rules():
    lib = O.restated_lib()
    assert lib.g4o_round_f16(1.0) == 1.0
    assert lib.g4o_round_f16(1.0 + 2 ** -11) == 1.0           # ties to even
    assert lib.g4o_round_f16(1.0 + 3 * 2 ** -11) == 1.0 + 2 ** -9
    assert lib.g4o_round_f16(3.0e-5) == 0.0                    # below the smallest normal half
    assert lib.g4o_round_f16(70000.0) == float("inf")


@pytest.mark.parametrize("tag,centered", [("baseline", False), ("centered", True)])
def test_restated_forward_matches_reference_golden(config0, tag, centered):
    path = config0["target_centered" if centered else "target"]
    from g4dense_b200 import container as C
    assert hashlib.sha256(Path(path).read_bytes()).hexdigest() == GOLDEN[f"container_sha256_{tag}"]
    g = GOLDEN[f"logits_{tag}"]
    m = O.RestatedModel(path)
    for p, (tok, want) in enumerate(zip(g["tokens"], g["positions"])):
        logits = m.forward(tok, p)
        assert hashlib.sha256(logits.tobytes()).hexdigest() == want["sha256"], f"position {p}"
        assert int(np.argmax(logits)) == want["argmax"]


@pytest.mark.parametrize("tag,centered", [("baseline", False), ("centered", True)])
def test_restated_decode_loop_matches_reference_golden(config0, tag, centered):
    tgt = config0["target_centered" if centered else "target"]
    drf = config0["draft_centered" if centered else "draft"]
    g = GOLDEN[f"streams_{tag}"]
    T = O.RestatedModel(tgt)
    for name, dpath in (("spec_k4", drf), ("self_draft_k4", tgt), ("no_spec", None)):
        D = O.RestatedModel(dpath) if dpath else None
        tokens, rounds = O.spec_generate(T, D, g["prompt"], 64, verify_width=5)
        assert tokens.tolist() == g[name]["tokens"], name
        assert [list(r) for r in rounds] == g[name]["rounds"], name


@pytest.mark.skipif(not O.reference_available(), reason="oracle/_ref not built")
def test_sampled_acceptance_matches_reference_rng():
    rng = np.random.default_rng(3)
    V = 512
    for trial in range(40):
        k = int(rng.integers(1, 6))
        tl = (rng.standard_normal((k + 1, V)) * 2).astype(np.float32)
        dl = (tl[:k] + rng.standard_normal((k, V)).astype(np.float32) * 0.5).astype(np.float32)
        drafts = [int(np.argmax(dl[i])) if rng.random() < 0.7 else int(rng.integers(0, V)) for i in range(k)]
        sp = O.Sampling(0.8, 1.0, 0, 1.0, 1, 77)
        a = O.evaluate_verification(drafts, tl, sp, base_seed=1000 + trial, draft_logits=dl)
        b = O.reference_evaluate_verification(drafts, tl, sp, base_seed=1000 + trial, draft_logits=dl)
        assert a == b, trial


@pytest.mark.skipif(not O.reference_available(), reason="oracle/_ref not built")
def test_sampled_token_draw_matches_reference():
    lib = O.restated_lib()
    ref = O.reference_lib()
    rng = np.random.default_rng(4)
    for trial in range(60):
        V = int(rng.integers(2, 3000))
        logits = (rng.standard_normal(V) * 3).astype(np.float32)
        t, p, k = [(0.8, 1.0, 0), (0.7, 0.9, 40), (1.2, 0.95, 256), (0.5, 1.0, 8)][trial % 4]
        sp = O.Sampling(t, p, k, 1.0, 1, 9)
        seed = int(rng.integers(1, 2 ** 62))
        a = lib.g4o_sample_token(logits.ctypes.data, V, sp, seed)
        b = ref.ref_sample_token(logits.ctypes.data, V, t, p, k, 1.0, 1, 9, seed)
        assert a == b, trial


GEOM31_GOLDEN = json.loads((Path(__file__).parent / "golden" / "geom31.json").read_text())


@pytest.mark.parametrize("tag,centered", [("baseline", False), ("centered", True)])
def test_restated_forward_matches_reference_on_31b_geometry(tmp_path, tag, centered):
    """Global layers (head_dim 512, 64 rotated pairs, V = raw K, GQA 4), GQA 2 sliding layers and
    a 48-key window wrapped twice by 120 positions: the restated forward pass reproduces the
    reference's CpuReferenceRunner logits bit for bit at every position."""
    from g4dense_b200 import container as C
    g = GEOM31_GOLDEN[tag]
    path = C.write_container(tmp_path / "g31.g4dense", C.GEOM31_TEST, seed=5, centered=centered)
    assert hashlib.sha256(path.read_bytes()).hexdigest() == g["container_sha256"]
    m = O.RestatedModel(path)
    for p, (tok, want) in enumerate(zip(g["tokens"], g["positions"])):
        logits = m.forward(tok, p)
        assert hashlib.sha256(logits.tobytes()).hexdigest() == want["sha256"], f"position {p}"
    assert len(g["positions"]) == 120


@pytest.mark.parametrize("key", ["pinned", "pinned_long"])
def test_restated_pinned_streams_match_reference_golden(config0, key):
    """The non-degenerate greedy cases the GPU tests compare exactly: the restated decode loop
    reproduces the reference's streams and round records, and the oracle's margins along the
    stream stay above the FP16 K/V rounding noise."""
    from g4dense_b200 import container as C
    g = GOLDEN[key]
    tgt, drf = config0["target_centered"], config0["draft_centered"]
    prompt = C.pinned_prompt(long=(key == "pinned_long"))
    assert prompt.tolist() == g["prompt"]
    T = O.RestatedModel(tgt)
    for name, dpath in (("no_spec", None), ("spec_k4", drf), ("self_draft_k4", tgt)):
        if name not in g:
            continue
        D = O.RestatedModel(dpath) if dpath else None
        tokens, rounds = O.spec_generate(T, D, prompt, g["n"], verify_width=g[name]["verify_width"] or 5)
        assert tokens.tolist() == g[name]["tokens"], name
        assert [list(r) for r in rounds] == g[name]["rounds"], name
    stream = g["no_spec"]["tokens"]
    assert len(set(stream)) >= 20, "the pinned stream must not be degenerate"
    assert min(O.greedy_margins(tgt, prompt, stream)) >= 0.09
    assert min(O.greedy_margins(drf, prompt, stream)) >= 0.02


def test_restated_sampled_streams_match_reference_golden(config0):
    """Temperature-0.8 speculative decoding with rejection sampling (src/speculator.cpp:71-122):
    the restated loop draws the same tokens and makes the same accept/reject decisions as the
    reference's, at verify widths 5 and 8, with a drafter that both accepts and rejects."""
    from g4dense_b200 import container as C
    g = GOLDEN["sampled"]
    assert hashlib.sha256(config0["near_draft"].read_bytes()).hexdigest() == g["container_sha256_near"]
    t, tp, tk, seed = g["params"]
    sp = O.Sampling(t, tp, tk, 1.0, 1, seed)
    T = O.RestatedModel(config0["target"])
    for name, dpath in (("near_w5", config0["near_draft"]), ("near_w8", config0["near_draft"]), ("no_spec", None)):
        D = O.RestatedModel(dpath) if dpath else None
        tokens, rounds = O.spec_generate(T, D, g["prompt"], g["n"], verify_width=g[name]["verify_width"] or 5,
                                         sampling=sp)
        assert tokens.tolist() == g[name]["tokens"], name
        assert [list(r) for r in rounds] == g[name]["rounds"], name
    acc = [r[1] for r in g["near_w5"]["rounds"] + g["near_w8"]["rounds"]]
    drafted = [r[0] for r in g["near_w5"]["rounds"] + g["near_w8"]["rounds"]]
    assert any(a < d for a, d in zip(acc, drafted)) and any(a == d for a, d in zip(acc, drafted))
