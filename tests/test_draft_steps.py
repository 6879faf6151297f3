"""Greedy drafting by the separate drafter on the device (g4dense_engine_draft_steps, the greedy case of
DraftRuntime::generate_draft_tokens, src/draft_runtime.cpp:46-95) against the CPU oracle.

Each drafter step is a one-row forward pass (src/runner.cpp:906-2059 as src/cpu_reference.cpp:245-672
computes it) whose argmax feeds the next step. The oracle (oracle/g4d_oracle.c, pinned to the
reference's CpuReferenceRunner) is teacher-forced with the GPU's own tokens, so every step's logits
are compared even if a near-tie lets the two chains part. Bars, as in test_engine.py: logits within
2e-2 of the row's max |logit| (K and V are rounded to FP16 before attention, so values on a rounding
boundary move by an FP16 ulp), and the drafted token equal to the oracle's argmax wherever the
oracle's top-2 margin clears that noise."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu
REL_TOL = 2e-2


def check_step(got_logits, tok, ref, where):
    d = np.abs(got_logits.astype(np.float64) - ref.astype(np.float64))
    scale = np.abs(ref).max()
    assert np.isfinite(got_logits).all(), where
    assert d.max() <= REL_TOL * scale, f"{where}: max |diff| {d.max():.3e} vs max |logit| {scale:.3f}"
    srt = np.sort(ref)[::-1]
    if srt[0] - srt[1] >= REL_TOL * scale:
        assert int(tok) == int(np.argmax(ref)), where
        return 1
    return 0


@pytest.fixture(scope="module")
def mid_pair(tmp_path_factory):
    from g4dense_b200 import container as C
    d = tmp_path_factory.mktemp("drafter")
    return (C.write_container(d / "t.g4dense", C.CONFIG0_TARGET, seed=0, centered=True),
            C.write_container(d / "d.g4dense", C.MID_TEST_DRAFT, seed=3, centered=True))


def test_draft_steps_match_oracle(built_lib, mid_pair):
    """200 chained steps from an empty cache, in calls of up to 64: the 64-key window wraps the
    ring (64 + 128 slots) and the attention spans 1..64 keys."""
    from g4dense_b200 import Engine
    tgt, drf = mid_pair
    e = Engine(target=tgt, draft=drf, draft_k=5, device=0)
    steps, first = 200, 11
    toks, logits = [], []
    tok, pos = first, 0
    while pos < steps:
        k = min(64, steps - pos)
        t, lg = e.draft_steps(tok, pos, k, vocab=4096)
        toks += [int(v) for v in t]
        logits += list(lg)
        tok, pos = int(t[-1]), pos + k
    e.close()
    ref = O.RestatedModel(drf)
    tok, checked = first, 0
    for s in range(steps):
        lg = ref.forward(tok, s)
        checked += check_step(logits[s], toks[s], lg, f"step {s}")
        tok = toks[s]  # teacher forcing with the GPU's own chain
    print(f"{steps} drafter steps compared with the oracle, {checked} tokens checked")
    assert checked >= steps * 3 // 4


def test_draft_steps_without_logits_match(built_lib, mid_pair):
    """The token-only path (no logits copied back) drafts the same tokens."""
    from g4dense_b200 import Engine
    tgt, drf = mid_pair
    a = Engine(target=tgt, draft=drf, draft_k=5, device=0)
    b = Engine(target=tgt, draft=drf, draft_k=5, device=0)
    ta, _ = a.draft_steps(7, 0, 48, vocab=4096)
    tb, lb = b.draft_steps(7, 0, 48)
    assert lb is None
    assert ta.tolist() == tb.tolist()
    a.close()
    b.close()


def test_draft_steps_rejects_bad_arguments(built_lib, mid_pair):
    from g4dense_b200 import Engine
    tgt, drf = mid_pair
    e = Engine(target=tgt, draft=drf, draft_k=5, device=0)
    with pytest.raises(RuntimeError):
        e.draft_steps(1, 0, 65)
    with pytest.raises(RuntimeError):
        e.draft_steps(1, 4090, 10)
    e.close()
    t = Engine(target=tgt, device=0)
    with pytest.raises(RuntimeError, match="drafter"):
        t.draft_steps(1, 0, 4)
    t.close()
