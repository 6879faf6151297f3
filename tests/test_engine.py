"""End-to-end parity of the B200 engine against the CPU oracle.

The oracle is oracle/g4d_oracle.c, pinned bit-for-bit to the reference's CpuReferenceRunner
by tests/test_oracle.py. Bars:
  * logits: max |gpu - oracle| <= 2e-2 of the row's max |logit| (BASELINE's relative 2e-2;
    the reference's own GPU test allows 0.5 absolute, tests/test_gpu_forward.cpp:142-200).
    Summation order alone moves values by ~1e-6 relative, but K and V are rounded to FP16
    before attention, so an element on an fp16 rounding boundary can land one ulp (2^-11)
    apart. The zero-mean test model amplifies that: in the oracle alone, FP16 vs FP32 KV
    moves its logits by up to 0.065. Argmax and top-5 order must agree wherever the margins
    exceed that noise (2e-2 of max |logit|);
  * greedy token streams and per-round (drafted, accepted, emitted) records: bit-identical
    on the BASELINE-distribution model (no KV rounding noise there). On the zero-mean model
    they must be identical up to the first position where the oracle's top-2 margin falls
    inside the rounding noise (< 0.05); a divergence is accepted only at such a near-tie,
    and round records are compared whenever the streams are identical.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu
REL_TOL = 2e-2


def engine(path, **kw):
    from g4dense_b200 import Engine
    return Engine(target=path, **kw)


def check_logits(got, ref, where):
    d = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    scale = np.abs(ref).max()
    assert np.isfinite(got).all(), where
    assert d.max() <= REL_TOL * scale, f"{where}: max |diff| {d.max():.3e} vs max |logit| {scale:.3f}"
    tie = REL_TOL * scale
    srt = np.sort(ref)[::-1]
    if srt[0] - srt[1] >= tie:
        assert int(np.argmax(got)) == int(np.argmax(ref)), where
        # Top-5 order, where every gap down to the 6th logit exceeds the noise bar.
        top = np.argsort(-ref, kind="stable")[:6]
        if np.all(np.diff(ref[top]) <= -tie):
            assert list(np.argsort(-got, kind="stable")[:5]) == list(top[:5]), where


@pytest.mark.parametrize("variant", ["target", "target_centered"])
def test_forward_batch_matches_oracle(built_lib, config0, variant):
    path = config0[variant]
    e = engine(path)
    ref = O.RestatedModel(path)
    toks = np.random.default_rng(11).integers(0, 4096, 40)
    want = [ref.forward(int(t), p) for p, t in enumerate(toks)]
    pos = 0
    for m in [1, 5, 16, 3, 15]:
        got = e.forward_batch(toks[pos:pos + m], pos, vocab=4096, all_positions=True)
        for i in range(m):
            check_logits(got[i], want[pos + i], f"{variant} position {pos + i} (batch {m})")
        pos += m
    e.close()


def test_bf16_kv_mode_matches_oracle(built_lib, config0):
    """Long-context mode: K/V rounded through bf16 (the oracle's BF16 KV mode); the attention
    kernel then runs its bf16 tensor-core variant."""
    path = config0["target"]
    e = engine(path, kv_bf16=True)
    ref = O.RestatedModel(path, kv_mode=O.KV_BF16)
    toks = np.random.default_rng(13).integers(0, 4096, 24)
    want = [ref.forward(int(t), p) for p, t in enumerate(toks)]
    pos = 0
    for m in [16, 1, 7]:
        got = e.forward_batch(toks[pos:pos + m], pos, vocab=4096, all_positions=True)
        for i in range(m):
            check_logits(got[i], want[pos + i], f"bf16 KV position {pos + i} (batch {m})")
        pos += m
    e.close()


@pytest.mark.parametrize("variant", ["baseline", "centered"])
def test_31b_attention_geometry_matches_oracle(built_lib, geom31, variant):
    """head_dim 256 / 512, GQA 2 and 4, a sliding window shorter than the context (ring wrap)
    and a full-attention layer long enough that every key split spans several tiles."""
    path = geom31[variant]
    e = engine(path, max_context=512)
    ref = O.RestatedModel(path, max_ctx=512)
    toks = np.random.default_rng(14).integers(0, 4096, 330)
    want = [ref.forward(int(t), p) for p, t in enumerate(toks)]
    pos = 0
    for m in [16] * 18 + [5, 1, 9, 16, 11]:
        got = e.forward_batch(toks[pos:pos + m], pos, vocab=4096, all_positions=True)
        for i in range(m):
            check_logits(got[i], want[pos + i], f"{variant} position {pos + i} (batch {m})")
        pos += m
    assert pos == len(toks)
    e.close()


def test_31b_geometry_bf16_kv(built_lib, geom31):
    """Long-context mode (bf16 K/V, three-term bf16 query/probability splits) on the 31B
    attention geometry: head_dim 512 with its head-dimension-split scores, GQA 4, a wrapped
    sliding ring. BASELINE-distribution weights."""
    path = geom31["baseline"]
    e = engine(path, max_context=512, kv_bf16=True)
    ref = O.RestatedModel(path, max_ctx=512, kv_mode=O.KV_BF16)
    toks = np.random.default_rng(15).integers(0, 4096, 200)
    want = [ref.forward(int(t), p) for p, t in enumerate(toks)]
    pos = 0
    for m in [16] * 10 + [9, 1, 5, 16, 9]:
        got = e.forward_batch(toks[pos:pos + m], pos, vocab=4096, all_positions=True)
        for i in range(m):
            check_logits(got[i], want[pos + i], f"bf16 KV position {pos + i} (batch {m})")
        pos += m
    assert pos == len(toks)
    e.close()


def test_batched_rows_equal_sequential(built_lib, config0):
    """tests/test_gpu_forward.cpp:205-260 / test_context_dependence.cpp: a batch of M rows
    computes what M single-row passes compute."""
    path = config0["target_centered"]
    toks = np.random.default_rng(12).integers(0, 4096, 9)
    a = engine(path)
    batched = a.forward_batch(toks, 0, vocab=4096, all_positions=True)
    b = engine(path)
    seq = np.stack([b.forward_batch(toks[i:i + 1], i, vocab=4096)[0] for i in range(len(toks))])
    for i in range(len(toks)):
        check_logits(batched[i], seq[i], f"row {i}")
    # On the BASELINE-distribution model the FP16 rounding noise vanishes: rows agree closely.
    path = config0["target"]
    batched = engine(path).forward_batch(toks, 0, vocab=4096, all_positions=True)
    e = engine(path)
    seq = np.stack([e.forward_batch(toks[i:i + 1], i, vocab=4096)[0] for i in range(len(toks))])
    assert np.abs(batched - seq).max() <= 1e-4


@pytest.mark.parametrize("tag", ["baseline", "centered"])
def test_greedy_streams_match_oracle(built_lib, config0, tag):
    sfx = "_centered" if tag == "centered" else ""
    tgt, drf = config0["target" + sfx], config0["draft" + sfx]
    prompt = np.random.default_rng(0).integers(0, 4096, 32)
    T = O.RestatedModel(tgt)
    margins = None
    for name, dpath in (("no_spec", None), ("spec_k4", drf), ("self_draft_k4", tgt)):
        D = O.RestatedModel(dpath) if dpath else None
        want_tokens, want_rounds = O.spec_generate(T, D, prompt, 64, verify_width=5)
        if margins is None:
            margins = O.greedy_margins(tgt, prompt, want_tokens)
        e = engine(tgt, draft=dpath, draft_k=5 if dpath else 0)
        got = e.generate(prompt, 64)
        if tag == "baseline":
            # No KV rounding noise on this model: streams are bit-identical, full stop.
            assert got.tolist() == want_tokens.tolist(), f"{tag}/{name} tokens"
        n = O.check_stream(got, want_tokens, margins)
        if n == len(want_tokens):
            assert e.rounds() == want_rounds, f"{tag}/{name} rounds"
        e.close()


def test_spec_streams_match_oracle_k8(built_lib, config0):
    """BASELINE config 4's k = 8 (verify width 9), wider than the reference's cap of 8."""
    tgt = config0["target_centered"]
    prompt = np.random.default_rng(1).integers(0, 4096, 20)
    want_tokens, want_rounds = O.spec_generate(O.RestatedModel(tgt), O.RestatedModel(tgt), prompt, 40, verify_width=9)
    e = engine(tgt, draft=tgt, draft_k=9)
    got = e.generate(prompt, 40)
    if O.check_stream(got, want_tokens, O.greedy_margins(tgt, prompt, want_tokens)) == len(want_tokens):
        assert e.rounds() == want_rounds
    e.close()


def test_replay_drafter_acceptance_sweep(built_lib, config0):
    """Config 3's oracle drafter: replaying the target's own greedy stream is always accepted;
    a 100% mismatch rate is never accepted and trips the adaptive gate after 24 drafts."""
    tgt, drf = config0["target_centered"], config0["draft_centered"]
    prompt = np.random.default_rng(0).integers(0, 4096, 32)
    stream, _ = O.spec_generate(O.RestatedModel(tgt), None, prompt, 60)
    margins = O.greedy_margins(tgt, prompt, stream)
    e = engine(tgt, draft=drf, draft_k=5)
    e.set_decode_options(replay=stream, mismatch_rate=0.0, mismatch_seed=3)
    if O.check_stream(e.generate(prompt, 60), stream, margins) == len(stream):
        assert all(r[1] == r[0] for r in e.rounds()[:-1])
    e.set_decode_options(replay=stream, mismatch_rate=1.0, mismatch_seed=3)
    if O.check_stream(e.generate(prompt, 60), stream, margins) == len(stream):
        rounds = e.rounds()
        assert all(r[1] == 0 for r in rounds) and len(rounds) == 6
    want = O.spec_generate(O.RestatedModel(tgt), O.RestatedModel(drf), prompt, 60, verify_width=5,
                           replay_stream=stream, mismatch_rate=0.25, mismatch_seed=9)
    e.set_decode_options(replay=stream, mismatch_rate=0.25, mismatch_seed=9)
    if O.check_stream(e.generate(prompt, 60), want[0], margins) == len(stream):
        assert e.rounds() == want[1]
    e.close()


def test_sampled_generation_is_seeded(built_lib, config0):
    tgt, drf = config0["target_centered"], config0["draft_centered"]
    prompt = np.random.default_rng(3).integers(0, 4096, 16)
    e = engine(tgt, draft=drf, draft_k=5)
    a = e.generate(prompt, 24, temperature=0.8, seed=5)
    b = e.generate(prompt, 24, temperature=0.8, seed=5)
    assert a.tolist() == b.tolist() and len(a) == 24
    e.close()


def test_callback_stop_and_telemetry(built_lib, config0):
    from g4dense_b200.api import lib
    e = engine(config0["target_centered"])
    seen = []
    out = e.generate(np.arange(10), 50, callback=lambda t: seen.append(t) or len(seen) < 3)
    assert len(out) == 3 and seen == out.tolist()
    assert lib().g4dense_engine_last_stop_reason(e.h) == 2
    tel = e.telemetry()
    for key in ("tps", "ttft_ms", "speculative_acceptance_rate", "total_tokens_generated", "kv_cache_mb"):
        assert key in tel
    assert lib().g4dense_engine_generate(e.h, b"hello", 4) is None
    assert b"tokenizer" in lib().g4dense_engine_last_error()
    e.close()


def _prefill_then_verify(e, ref_rows, toks, chunks, where):
    """Feeds `toks` in `chunks`: chunks above 16 rows are tensor-core prefill passes (last row's
    logits checked), the rest verify passes (every row checked)."""
    pos = 0
    for m in chunks:
        if m > 16:
            got = e.forward_batch(toks[pos:pos + m], pos, vocab=4096, all_positions=False)
            check_logits(got[0], ref_rows[pos + m - 1], f"{where} prefill chunk at {pos} (rows {m}), last row")
        else:
            got = e.forward_batch(toks[pos:pos + m], pos, vocab=4096, all_positions=True)
            for i in range(m):
                check_logits(got[i], ref_rows[pos + i], f"{where} position {pos + i} (batch {m})")
        pos += m
    assert pos == len(toks)


@pytest.mark.parametrize("variant", ["target", "target_centered"])
def test_prefill_chunks_match_oracle(built_lib, config0, variant):
    """Tensor-core prefill chunks (17..128 rows) against the oracle: the chunk's last-row logits,
    then verify passes that read the K/V the chunks wrote."""
    path = config0[variant]
    e = engine(path)
    ref = O.RestatedModel(path)
    toks = np.random.default_rng(21).integers(0, 4096, 330)
    want = [ref.forward(int(t), p) for p, t in enumerate(toks)]
    _prefill_then_verify(e, want, toks, [128, 17, 100, 64, 16, 5], variant)
    e.close()


def test_prefill_chunks_bf16_kv(built_lib, config0):
    path = config0["target"]
    e = engine(path, kv_bf16=True)
    ref = O.RestatedModel(path, kv_mode=O.KV_BF16)
    toks = np.random.default_rng(22).integers(0, 4096, 200)
    want = [ref.forward(int(t), p) for p, t in enumerate(toks)]
    _prefill_then_verify(e, want, toks, [128, 56, 16], "bf16 KV")
    e.close()


def test_prefill_chunks_31b_geometry(built_lib, geom31):
    """head_dim 256 / 512, GQA 2 and 4 and a 48-key sliding window far shorter than a 128-row
    chunk: the ring holds window + 128 slots so a chunk never overwrites a key it still reads.
    BASELINE-distribution weights only: over 400 positions the zero-mean model turns one-ulp
    FP16 K/V rounding differences into logit moves beyond 2e-2 on the verify path alone (seen
    from position ~100 with this sequence), so there it would test the rounding, not the kernels;
    the zero-mean model's prefill chunks are covered on config 0 above."""
    variant = "baseline"
    path = geom31[variant]
    e = engine(path, max_context=512)
    ref = O.RestatedModel(path, max_ctx=512)
    toks = np.random.default_rng(23).integers(0, 4096, 420)
    want = [ref.forward(int(t), p) for p, t in enumerate(toks)]
    _prefill_then_verify(e, want, toks, [128, 128, 97, 49, 16, 2], variant)
    e.close()


def test_long_prompt_streams_match_oracle(built_lib, config0):
    """A 300-token prompt is prefilled in tensor-core chunks (128, 128, then 44 rows as verify
    passes); the greedy streams that follow must still equal the oracle's bit for bit."""
    tgt, drf = config0["target"], config0["draft"]
    prompt = np.random.default_rng(24).integers(0, 4096, 300)
    T = O.RestatedModel(tgt)
    for name, dpath in (("no_spec", None), ("spec_k4", drf)):
        D = O.RestatedModel(dpath) if dpath else None
        want_tokens, want_rounds = O.spec_generate(T, D, prompt, 32, verify_width=5)
        e = engine(tgt, draft=dpath, draft_k=5 if dpath else 0)
        got = e.generate(prompt, 32)
        assert got.tolist() == want_tokens.tolist(), f"{name} tokens"
        assert e.rounds() == want_rounds, f"{name} rounds"
        e.close()
