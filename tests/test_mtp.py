"""MTP "assistant" drafter (.g4mtp; src/mtp_runner.cpp) against the oracle's restatement.

The reference's MTP runner exists only as Vulkan compute (no CPU path), so the oracle
(oracle/g4d_oracle.c g4o_mtp_draft) restates its steps and its parity is unpinned: it shares the
pinned forward-pass helpers (INT4 GEMV, RMSNorm, RoPE, attention) but no reference output checks
the MTP composition itself. The container is written by g4dense_b200.container with the
converter's layout (tools/convert_hf_assistant.py:114-176) and read by both sides.

Checks: the header and layout (CPU); per-step drafter logits and tokens against the oracle (GPU);
speculative decoding with the MTP drafter emits exactly the target's greedy stream (GPU).

The drafter reads the target's KV cache and final hidden state, so its inputs carry the
target's own forward-pass error, and a random zero-mean network amplifies that: with the
zero-mean target the drafter's step-0 logits differ by 2-15 % of their range while the target's
logits agree within 0.2-2 %. The logit parity test therefore drafts from the BASELINE-distribution
target (positive-mean weights), whose forward pass the GPU reproduces to 1e-5, with a zero-mean
drafter whose tokens do depend on its input. There the drafter's logits must agree within 1e-3
of their range and every drafted token must match. The zero-mean target is used where only
exact invariants are checked (speculative output equals the greedy stream).
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O

from test_engine import engine


@pytest.fixture(scope="module")
def mtp_pair(tmp_path_factory):
    from g4dense_b200 import container as C
    d = tmp_path_factory.mktemp("mtp")
    target = C.write_container(d / "target.g4dense", C.MTP_TEST_TARGET, seed=5, centered=True)
    spec = C.MtpSpec.for_target(C.MTP_TEST_TARGET)
    mtp = C.write_mtp_container(d / "assistant.g4mtp", spec, seed=6, centered=True)
    return target, mtp, spec


@pytest.fixture(scope="module")
def mtp_bias_target(tmp_path_factory):
    from g4dense_b200 import container as C
    d = tmp_path_factory.mktemp("mtp_bias")
    return C.write_container(d / "target.g4dense", C.MTP_TEST_TARGET, seed=5)


def test_mtp_container_layout(mtp_pair, tmp_path):
    from g4dense_b200 import container as C
    _, path, spec = mtp_pair
    raw = path.read_bytes()
    assert len(raw) % 4096 == 0 and raw[:4] == b"TM4G"
    m = O.RestatedMtp(path)
    info = np.zeros(12, np.uint32)
    m.lib.g4o_mtp_info(m.h, info.ctypes.data)
    assert info[:8].tolist() == [spec.num_layers, spec.backbone, spec.hidden, spec.intermediate, spec.vocab_size,
                                 spec.num_q_heads, spec.num_kv_heads, spec.head_dim]
    m.close()
    bad = bytearray(raw)
    bad[0] ^= 1
    (tmp_path / "bad.g4mtp").write_bytes(bad)
    with pytest.raises(RuntimeError, match="invalid header"):
        O.RestatedMtp(tmp_path / "bad.g4mtp")
    assert len(C.build_mtp_container(C.GEMMA4_31B_ASSISTANT.__class__(**{**C.GEMMA4_31B_ASSISTANT.__dict__,
                                                                           "vocab_size": 512, "hidden": 64,
                                                                           "intermediate": 128, "backbone": 128,
                                                                           "num_q_heads": 2, "num_kv_heads": 1,
                                                                           "head_dim": 64, "global_head_dim": 64,
                                                                           "global_kv_heads": 1}))) % 4096 == 0


def test_oracle_mtp_draft_is_deterministic(mtp_pair):
    target, path, _ = mtp_pair
    t = O.RestatedModel(target)
    toks = np.random.default_rng(1).integers(0, 4096, 20)
    hid = None
    for p, tok in enumerate(toks):
        _, hid = t.forward(int(tok), p, want_hidden=True)
    m = O.RestatedMtp(path)
    a, la = m.draft(t, hid, 7, len(toks) + 1, 3)
    b, lb = m.draft(t, hid, 7, len(toks) + 1, 3)
    assert a.tolist() == b.tolist() and np.array_equal(la, lb)
    assert np.isfinite(la).all() and (a < 4096).all()


def _oracle_state(target, toks):
    t = O.RestatedModel(target)
    hid = None
    for p, tok in enumerate(toks):
        _, hid = t.forward(int(tok), p, want_hidden=True)
    return t, hid


@pytest.mark.gpu
@pytest.mark.parametrize("n_prompt,chunks", [(12, [12]), (40, [40]), (100, [100]), (90, [80, 10])])
def test_mtp_draft_matches_oracle(built_lib, mtp_pair, mtp_bias_target, n_prompt, chunks):
    """Prompts shorter and longer than the 64-key window, fed as one prefill chunk (>16 rows:
    the hidden state is row 0) or ending with a verify-width pass (row M - 1)."""
    _, path, _ = mtp_pair
    target = mtp_bias_target
    toks = np.random.default_rng(n_prompt).integers(0, 4096, n_prompt)
    e = engine(target, draft=path)
    pos = 0
    for m in chunks:
        e.forward_batch(toks[pos:pos + m], pos)
        pos += m
    row = 0 if chunks[-1] > 16 else chunks[-1] - 1
    seed_tok = int(toks[-1]) ^ 5
    k = 4
    got_t, got_l = e.mtp_draft(seed_tok, n_prompt + 1, row, k, 4096)
    t, hid = _oracle_state(target, toks)
    m = O.RestatedMtp(path)
    want_t, want_l = m.draft(t, hid, seed_tok, n_prompt + 1, k)
    for s in range(k):
        scale = np.abs(want_l[s]).max()
        err = np.abs(got_l[s].astype(np.float64) - want_l[s]).max()
        assert err <= 1e-3 * scale, f"MTP step {s} (prompt {n_prompt}): max |diff| {err:.3e} vs {scale:.3f}"
        assert got_t[s] == want_t[s], s
    e.close()


@pytest.mark.gpu
@pytest.mark.parametrize("k", [2, 5])
def test_spec_decode_with_mtp_equals_greedy(built_lib, mtp_pair, k):
    target, path, _ = mtp_pair
    prompt = np.random.default_rng(3).integers(0, 4096, 30)
    plain = engine(target)
    want = plain.generate(prompt, 48)
    plain.close()
    e = engine(target, draft=path, draft_k=k)
    got = e.generate(prompt, 48)
    assert got.tolist() == want.tolist()
    assert len(e.rounds()) > 0
    e.close()


@pytest.mark.gpu
def test_sampled_spec_decode_with_mtp_is_seeded(built_lib, mtp_pair):
    target, path, _ = mtp_pair
    prompt = np.random.default_rng(4).integers(0, 4096, 24)
    e = engine(target, draft=path, draft_k=4)
    a = e.generate(prompt, 24, temperature=0.8, top_k=40, top_p=0.9, seed=2)
    b = e.generate(prompt, 24, temperature=0.8, top_k=40, top_p=0.9, seed=2)
    assert a.tolist() == b.tolist() and len(a) == 24
    e.close()
