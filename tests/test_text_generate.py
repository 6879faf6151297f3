"""The engine's text entry points (g4dense_engine_generate / _generate_ex / _generate_text) against
the reference path on the same inputs.

The expected stream is built from reference code: the reference's own tokenizer (oracle/_ref,
else the restatement pinned to its golden vectors) applies the chat template and encodes the
prompt, the restated runner (oracle/g4d_oracle.c) decodes it on the same container, generation
ends after the first tokenizer stop id (src/runner.cpp:2111-2118, 2336), and the response is the
concatenation of decode_single pieces (src/c_api.cpp:100-105). Tokens, the response and every
callback piece must be identical. The prompts (g4dense_b200.synth_tokenizer) keep the oracle's
greedy top-2 margins at or above 0.05 along their streams (tests/test_tokenizer.py checks this on
the CPU), so an exact comparison tests the engine, not a near-tie.
"""
from __future__ import annotations

import ctypes
import os
import shutil

import numpy as np
import pytest

from oracle import oracle as O
from oracle import tokenizer_oracle as TO

pytestmark = pytest.mark.gpu

from g4dense_b200.synth_tokenizer import RAW_PROMPTS, STOP_PROMPT


@pytest.fixture(scope="module")
def tokp(tmp_path_factory):
    from g4dense_b200 import synth_tokenizer as S
    return S.write_synthetic_tokenizer(tmp_path_factory.mktemp("text") / "tokenizer.json")


def ref_tokenizer(path):
    return O.ReferenceTokenizer(path) if O.reference_available() else TO.Tokenizer(path)


def expected(target, tokp, prompt, n, chat=True, sampling=None, draft=None, width=5):
    R = ref_tokenizer(tokp)
    if chat:
        ids = R.encode(R.chat_template([("user", prompt)]), False)
    else:
        ids = R.encode(prompt.encode(), True)
    toks, _ = O.spec_generate(O.RestatedModel(target), O.RestatedModel(draft) if draft else None, ids, n,
                              verify_width=width, sampling=sampling)
    toks = toks.tolist()
    stops = R.stop_ids() if hasattr(R, "stop_ids") and callable(R.stop_ids) else R.stop_ids
    cut = next((i for i, t in enumerate(toks) if t in stops), None)
    if cut is not None:
        toks = toks[:cut + 1]
    return toks, [R.decode_single(t) for t in toks], cut is not None


def options(max_tokens, temperature=0.0, top_p=1.0, top_k=0):
    from g4dense_b200.api import GenOptions, lib
    o = GenOptions()
    lib().g4dense_options_default(ctypes.byref(o))
    o.max_tokens, o.temperature, o.top_p, o.top_k = max_tokens, temperature, top_p, top_k
    return o


def test_generate_ex_greedy_matches_reference(built_lib, config0, tokp):
    from g4dense_b200.api import TOKEN_CB, Engine, lib
    tgt = config0["target_centered"]
    e = Engine(tgt, tokenizer_path=tokp)
    for prompt in (STOP_PROMPT,):
        want, pieces, stopped = expected(tgt, tokp, prompt, 48)
        assert stopped, "the case no longer reaches a stop id"
        seen = []
        cb = TOKEN_CB(lambda u, i, t, d: seen.append((i, t, d)) or 1)
        o = options(48)
        r = lib().g4dense_engine_generate_ex(e.h, prompt.encode(), ctypes.byref(o), cb, None)
        assert r is not None, lib().g4dense_engine_last_error()
        assert e.tokens().tolist() == want
        assert seen == [(i, t, p) for i, (t, p) in enumerate(zip(want, pieces))]
        assert r == b"".join(pieces)
        assert lib().g4dense_engine_last_stop_reason(e.h) == 1
        print(f"{prompt!r}: {len(want)} tokens, stop id {want[-1]}, response {r[:60]!r}")
    e.close()


def test_generate_default_sampling_matches_reference(built_lib, config0, tokp):
    """g4dense_engine_generate: temperature 0.2, top_p 0.95, top_k 64, no seed (the per-position
    seeds of seed_for), drawn on the device. The stream is compared token for token over 40
    tokens; a longer sampled stream can part from the CPU oracle's where a temperature-0.2 draw
    falls within the logits' tolerance (2e-2 of the row maximum) of a bucket edge, so the second
    call checks only that the response is the pieces of the emitted tokens."""
    from g4dense_b200.api import Engine, lib
    tgt = config0["target_centered"]
    e = Engine(tgt, tokenizer_path=tokp)
    want, pieces, _ = expected(tgt, tokp, "kato rien", 40, sampling=O.Sampling(0.2, 0.95, 64, 1.0, 0, 0))
    r = lib().g4dense_engine_generate(e.h, b"kato rien", 40)
    assert r is not None, lib().g4dense_engine_last_error()
    assert e.tokens().tolist() == want and r == b"".join(pieces)
    R = ref_tokenizer(tokp)
    r = lib().g4dense_engine_generate(e.h, STOP_PROMPT.encode(), 0)  # max_tokens <= 0: 512
    toks = e.tokens().tolist()
    assert r == b"".join(R.decode_single(t) for t in toks)
    stops = R.stop_ids() if callable(R.stop_ids) else R.stop_ids
    assert (toks[-1] in stops) == (lib().g4dense_engine_last_stop_reason(e.h) == 1)
    assert len(toks) == 512 or toks[-1] in stops
    e.close()


def test_generate_text_raw_prompt_speculative(built_lib, config0, tokp):
    """use_chat_template = 0 (<bos> + raw text), with the separate drafter at verify width 5."""
    from g4dense_b200.api import Engine
    tgt, drf = config0["target_centered"], config0["draft_centered"]
    e = Engine(tgt, draft=drf, draft_k=5, tokenizer_path=tokp)
    for prompt in RAW_PROMPTS:
        want, pieces, _ = expected(tgt, tokp, prompt, 40, chat=False, draft=drf, width=5)
        got_pieces = []
        r = e.generate_text(prompt, use_chat_template=False, max_tokens=40,
                            callback=lambda t, d: got_pieces.append(d) or True)
        assert e.tokens().tolist() == want and r == b"".join(pieces) and got_pieces == pieces
        assert e.stats()["rounds"] > 0
    e.close()


def test_callback_stop_and_cancel(built_lib, config0, tokp):
    from g4dense_b200.api import Engine, lib
    e = Engine(config0["target_centered"], tokenizer_path=tokp)
    seen = []
    r = e.generate_text("kato", max_tokens=30, callback=lambda t, d: seen.append(d) or len(seen) < 3)
    assert len(e.tokens()) == 3 and r == b"".join(seen)
    assert lib().g4dense_engine_last_stop_reason(e.h) == 2
    e.close()


def test_tokenizer_discovery(built_lib, config0, tokp, tmp_path):
    from g4dense_b200.api import Engine, lib
    # none: text calls fail the way the reference's runner does
    e = Engine(preset="config0-target")
    assert e.tokenizer() is None
    assert lib().g4dense_engine_generate(e.h, b"hi", 4) is None
    assert b"Tokenizer is not loaded" in lib().g4dense_engine_last_error()
    e.close()
    # tokenizer.json beside the container
    shutil.copy(config0["target_centered"], tmp_path / "model.g4dense")
    shutil.copy(tokp, tmp_path / "tokenizer.json")
    e = Engine(tmp_path / "model.g4dense")
    t = e.tokenizer()
    assert t is not None and t.special_ids()["vocab_size"] == 4096 and t.stop_ids() == [1, 106, 50]
    assert t.encode("kato") == ref_tokenizer(tokp).encode(b"kato")
    e.close()
    # $G4DENSE_TOKENIZER
    os.environ["G4DENSE_TOKENIZER"] = str(tokp)
    try:
        e = Engine(preset="config0-target")
        assert e.tokenizer() is not None
        e.close()
    finally:
        del os.environ["G4DENSE_TOKENIZER"]
    # an explicit path that does not exist is an error at creation
    with pytest.raises(RuntimeError, match="Failed to open tokenizer"):
        Engine(preset="config0-target", tokenizer_path=tmp_path / "missing.json")
