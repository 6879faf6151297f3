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
  * greedy token streams and per-round (drafted, accepted, emitted) records: identical, with
    plain asserts. The BASELINE-distribution model's greedy stream is one token repeated, so
    the streams that carry the check run the zero-mean model on the pinned prompts
    (container.PINNED_*): seeds chosen so that the oracle's top-2 margins along the whole stream
    stay at least twice the FP16 K/V rounding noise, pinned to the reference's own CPU loop by
    tests/golden/config0.json. Every test prints how many tokens and rounds it compared;
  * sampled speculative decoding (temperature 0.8, rejection sampling): tokens and round
    records identical to the oracle's, on the BASELINE-distribution target (which the GPU
    reproduces to ~1e-5) with a drafter that both accepts and rejects.
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


def _compare(got, got_rounds, want, want_rounds, where):
    """Plain equality of streams and round records, reporting what was compared."""
    assert got.tolist() == want.tolist(), f"{where}: tokens differ at {next((i for i, (a, b) in enumerate(zip(got, want)) if a != b), min(len(got), len(want)))}"
    assert got_rounds == want_rounds, f"{where}: rounds {got_rounds} != {want_rounds}"
    print(f"{where}: compared {len(want)} tokens and {len(want_rounds)} rounds "
          f"({sum(r[1] for r in want_rounds)}/{sum(r[0] for r in want_rounds)} drafts accepted)")


@pytest.mark.parametrize("tag", ["baseline", "pinned"])
def test_greedy_streams_match_oracle(built_lib, config0, tag):
    from g4dense_b200 import container as C
    sfx = "_centered" if tag == "pinned" else ""
    tgt, drf = config0["target" + sfx], config0["draft" + sfx]
    prompt = C.pinned_prompt() if tag == "pinned" else np.random.default_rng(0).integers(0, 4096, 32)
    T = O.RestatedModel(tgt)
    for name, dpath in (("no_spec", None), ("spec_k4", drf), ("self_draft_k4", tgt)):
        D = O.RestatedModel(dpath) if dpath else None
        want_tokens, want_rounds = O.spec_generate(T, D, prompt, 64, verify_width=5)
        e = engine(tgt, draft=dpath, draft_k=5 if dpath else 0)
        got = e.generate(prompt, 64)
        _compare(got, e.rounds(), want_tokens, want_rounds, f"{tag}/{name}")
        e.close()
    if tag == "pinned":
        assert len(set(want_tokens.tolist())) >= 20


@pytest.mark.parametrize("drafter", ["self", "draft"])
def test_spec_streams_match_oracle_k8(built_lib, config0, drafter):
    """BASELINE config 4's k = 8 (verify width 9), wider than the reference's cap of 8."""
    from g4dense_b200 import container as C
    tgt = config0["target_centered"]
    dpath = tgt if drafter == "self" else config0["draft_centered"]
    prompt = C.pinned_prompt()
    want_tokens, want_rounds = O.spec_generate(O.RestatedModel(tgt), O.RestatedModel(dpath), prompt, 48,
                                               verify_width=9)
    e = engine(tgt, draft=dpath, draft_k=9)
    got = e.generate(prompt, 48)
    _compare(got, e.rounds(), want_tokens, want_rounds, f"k8/{drafter}")
    e.close()


def test_replay_drafter_acceptance_sweep(built_lib, config0):
    """Config 3's oracle drafter: replaying the target's own greedy stream is always accepted;
    a 100% mismatch rate is never accepted and trips the adaptive gate after 24 drafts; at 25%
    the rounds mix accepts and rejects exactly as the oracle's do."""
    from g4dense_b200 import container as C
    tgt, drf = config0["target_centered"], config0["draft_centered"]
    prompt = C.pinned_prompt()
    T = O.RestatedModel(tgt)
    stream, _ = O.spec_generate(T, None, prompt, 60)
    e = engine(tgt, draft=drf, draft_k=5)
    for rate, seed in ((0.0, 3), (1.0, 3), (0.25, 9), (0.5, 4)):
        want = O.spec_generate(T, O.RestatedModel(drf), prompt, 60, verify_width=5, replay_stream=stream,
                               mismatch_rate=rate, mismatch_seed=seed)
        e.set_decode_options(replay=stream, mismatch_rate=rate, mismatch_seed=seed)
        got = e.generate(prompt, 60)
        _compare(got, e.rounds(), want[0], want[1], f"replay rate {rate}")
        assert got.tolist() == stream.tolist()
        rounds = want[1]
        if rate == 0.0:
            assert all(r[1] == r[0] for r in rounds[:-1])
        if rate == 1.0:
            assert all(r[1] == 0 for r in rounds) and len(rounds) == 6
        if rate == 0.25:
            assert any(0 < r[1] < r[0] for r in rounds)
    e.close()


def test_sampled_spec_matches_oracle(built_lib, config0):
    """Temperature-0.8 speculative decoding (the config-4 sampled mode): drafts drawn with the
    reference's per-step seeds, accepted or rejected by the ratio test with the mt19937_64
    draw, residual draws on rejection (src/speculator.cpp:71-122). Tokens and (drafted, accepted,
    emitted) records equal the oracle's at verify widths 5, 8 and 9; widths 5 and 8 also equal
    the reference's own loop (tests/golden/config0.json)."""
    import json
    from pathlib import Path
    g = json.loads((Path(__file__).parent / "golden" / "config0.json").read_text())["sampled"]
    t, tp, tk, seed = g["params"]
    sp = O.Sampling(t, tp, tk, 1.0, 1, seed)
    tgt, near = config0["target"], config0["near_draft"]
    T = O.RestatedModel(tgt)
    mixed = False
    for width in (5, 8, 9):
        want_tokens, want_rounds = O.spec_generate(T, O.RestatedModel(near), g["prompt"], g["n"], verify_width=width,
                                                   sampling=sp)
        if f"near_w{width}" in g:
            assert want_tokens.tolist() == g[f"near_w{width}"]["tokens"]
        e = engine(tgt, draft=near, draft_k=width)
        got = e.generate(g["prompt"], g["n"], temperature=t, top_p=tp, top_k=tk, seed=seed)
        _compare(got, e.rounds(), want_tokens, want_rounds, f"sampled width {width}")
        mixed |= any(r[1] < r[0] for r in want_rounds)
        e.close()
    assert mixed, "no round rejected a draft: the case does not exercise the residual draw"


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
    for key in ("tps", "ttft_ms", "speculative_acceptance_rate", "total_tokens_generated", "kv_cache_mb",
                "pinned_layers", "lm_head_mb", "draft_k", "context_tokens"):
        assert key in tel
    assert lib().g4dense_engine_generate(e.h, b"hello", 4) is None
    assert b"tokenizer" in lib().g4dense_engine_last_error().lower()
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
    passes); the greedy streams and round records that follow must equal the oracle's."""
    from g4dense_b200 import container as C
    tgt, drf = config0["target_centered"], config0["draft_centered"]
    prompt = C.pinned_prompt(long=True)
    T = O.RestatedModel(tgt)
    for name, dpath in (("no_spec", None), ("spec_k4", drf)):
        D = O.RestatedModel(dpath) if dpath else None
        want_tokens, want_rounds = O.spec_generate(T, D, prompt, C.PINNED_LONG_TOKENS, verify_width=5)
        e = engine(tgt, draft=dpath, draft_k=5 if dpath else 0)
        got = e.generate(prompt, C.PINNED_LONG_TOKENS)
        _compare(got, e.rounds(), want_tokens, want_rounds, f"long prompt/{name}")
        e.close()
