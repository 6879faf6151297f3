"""The engine's tokenizer (g4dense_tokenizer_*; csrc/tokenizer.cpp) against the reference's.

Three implementations are compared on the same inputs:
  * the engine's C++ tokenizer, through its C ABI;
  * the reference's own Tokenizer / IncrementalDetokenizer / StreamingStopMatcher / utf8_repair
    (src/tokenizer.cpp, src/detokenizer.cpp compiled unmodified into oracle/_ref), live where it
    is built and through the golden vectors it produced (tests/golden/tokenizer.json) everywhere;
  * the Python restatement in oracle/tokenizer_oracle.py, pinned to those golden vectors.
The vocabulary is the synthetic Gemma-4-style tokenizer.json of g4dense_b200.synth_tokenizer.
The cases the reference's own tests assert (tests/test_tokenizer.cpp, tests/test_detokenizer.cpp)
are restated at the end. All of this is host code: no GPU is needed.
"""
from __future__ import annotations

import hashlib
import json
import time
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O
from oracle import tokenizer_oracle as TO

GOLDEN = json.loads((Path(__file__).parent / "golden" / "tokenizer.json").read_text())


@pytest.fixture(scope="module")
def tok_paths(tmp_path_factory):
    from g4dense_b200 import synth_tokenizer as S
    d = tmp_path_factory.mktemp("tok")
    p = S.write_synthetic_tokenizer(d / "pair.json", merges_as_pairs=True)
    j = S.write_synthetic_tokenizer(d / "joined.json", merges_as_pairs=False)
    assert hashlib.sha256(p.read_bytes()).hexdigest() == GOLDEN["sha256"]["pair"], \
        "the synthetic tokenizer.json changed: regenerate tests/golden/tokenizer.json"
    assert hashlib.sha256(j.read_bytes()).hexdigest() == GOLDEN["sha256"]["joined"]
    return {"pair": p, "joined": j}


@pytest.fixture(scope="module")
def engine_tok(built_lib, tok_paths):
    from g4dense_b200.api import Tokenizer
    return Tokenizer(tok_paths["pair"])


def _check_against_golden(T, stream_fn, stop_fn, repair_fn, chat_fn, ids_fn):
    g = GOLDEN["pair"]
    for i, c in enumerate(g["encode"]):
        got = T.encode(bytes.fromhex(c["text"]), c["add_bos"])
        assert got == c["ids"], f"encode case {i}: {bytes.fromhex(c['text'])!r}"
    for i, c in enumerate(g["decode"]):
        assert T.decode(c["ids"], c["skip_special"]).hex() == c["out"], f"decode case {i}"
    ds = g["decode_single"]
    h0, h1 = hashlib.sha256(), hashlib.sha256()
    for t in range(ds["ids"]):
        h0.update(T.decode_single(t, False) + b"\x00")
        h1.update(T.decode_single(t, True) + b"\x00")
    assert h0.hexdigest() == ds["sha256_keep_special"] and h1.hexdigest() == ds["sha256_skip_special"]
    for t, piece in ds["samples"].items():
        assert T.decode_single(int(t), False).hex() == piece
    for t in range(ds["ids"]):
        assert T.byte_value(t) == g["byte_values"].get(str(t)), t
    assert [t for t in range(ds["ids"]) if T.is_special(t)] == g["special"]
    for i, c in enumerate(g["stream"]):
        assert [p.hex() for p in stream_fn(c["ids"], c["skip_special"])] == c["pushes"], f"stream case {i}"
    for i, c in enumerate(g["stop"]):
        outs, stopped, matched = stop_fn([bytes.fromhex(s) for s in c["stops"]],
                                         [bytes.fromhex(x) for x in c["chunks"]])
        assert ([o.hex() for o in outs], stopped, matched.hex()) == (c["outs"], c["stopped"], c["matched"]), \
            f"stop case {i}"
    for i, c in enumerate(g["utf8_repair"]):
        out, used = repair_fn(bytes.fromhex(c["in"]), c["flush_all"])
        assert (out.hex(), used) == (c["out"], c["consumed"]), f"utf8_repair case {i}"
    for i, c in enumerate(g["chat"]):
        got = chat_fn(c["arch"], c["messages"])
        assert got == c["out"], f"chat case {i}: {got} != {c['out']}"
    for arch in (0, 1):
        assert ids_fn(arch) == g[f"ids_arch{arch}"]


# ---------------------------------------------------------------- the restatement, pinned

def test_restatement_matches_reference_golden(tok_paths):
    """oracle/tokenizer_oracle.py reproduces every golden vector of the reference's tokenizer."""
    T = TO.Tokenizer(tok_paths["pair"])

    def stream(ids, skip):
        d = TO.Detokenizer(T, skip)
        return [d.push(t) for t in ids] + [d.finish()]

    def stop(stops, chunks):
        m = TO.StopMatcher(stops)
        return [m.push(c) for c in chunks] + [m.finish()], m.stopped, m.matched

    def chat(arch, msgs):
        try:
            return TO.Tokenizer(tok_paths["pair"], arch).chat_template(msgs).hex()
        except ValueError as e:
            return {"error": str(e)}

    def ids(arch):
        A = TO.Tokenizer(tok_paths["pair"], arch)
        return {"bos": A.bos, "eos": A.eos, "pad": A.pad, "unk": A.unk, "end_of_turn": A.end_of_turn,
                "vocab_size": A.vocab_size, "stop": A.stop_ids}
    _check_against_golden(T, stream, stop, TO.utf8_repair, chat, ids)
    J = TO.Tokenizer(tok_paths["joined"])
    for c in GOLDEN["joined_encode"]:
        assert J.encode(bytes.fromhex(c["text"]), c["add_bos"]) == c["ids"]


# ---------------------------------------------------------------- the engine's tokenizer

def _engine_fns(T, path):
    from g4dense_b200 import api

    def stream(ids, skip):
        d = T.detokenizer(skip)
        return [d.push(int(t)) for t in ids] + [d.finish()]

    def stop(stops, chunks):
        m = api.StopMatcher(stops)
        return [m.push(c) for c in chunks] + [m.finish()], m.stopped, m.matched

    def chat(arch, msgs):
        A = api.Tokenizer(path, arch)
        try:
            return A.chat_template(msgs).hex()
        except RuntimeError as e:
            return {"error": str(e).split(": ", 1)[1]}

    def ids(arch):
        A = api.Tokenizer(path, arch)
        return {**A.special_ids(), "stop": A.stop_ids()}
    return stream, stop, api.utf8_repair, chat, ids


def test_engine_tokenizer_matches_reference_golden(engine_tok, tok_paths):
    _check_against_golden(engine_tok, *_engine_fns(engine_tok, tok_paths["pair"]))
    from g4dense_b200.api import Tokenizer
    J = Tokenizer(tok_paths["joined"])
    for c in GOLDEN["joined_encode"]:
        assert J.encode(bytes.fromhex(c["text"]), c["add_bos"]) == c["ids"]


@pytest.mark.skipif(not O.reference_available(), reason="oracle/_ref is not built")
def test_engine_tokenizer_matches_reference_live(engine_tok, tok_paths):
    """Fresh random cases (another seed, longer texts) against the reference's compiled tokenizer."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("mkg", Path(__file__).parent / "golden" / "make_tokenizer_golden.py")
    mkg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mkg)
    R = O.ReferenceTokenizer(tok_paths["pair"])
    enc, dec, stream, stop, repair = mkg.make_cases(seed=2024, n_encode=400, n_decode=200, n_stream=150, n_stop=150,
                                                    n_repair=150)
    rng = np.random.default_rng(7)
    enc += [(mkg.random_text(rng, int(rng.integers(300, 1200))), True) for _ in range(8)]
    for text, bos in enc:
        assert engine_tok.encode(text, bos) == R.encode(text, bos), text
    for ids, skip in dec:
        assert engine_tok.decode(ids, skip) == R.decode(ids, skip)
    fn_stream, fn_stop, fn_repair, _, _ = _engine_fns(engine_tok, tok_paths["pair"])
    for ids, skip in stream:
        assert fn_stream(ids, skip) == R.stream(ids, skip)
    for stops, chunks in stop:
        assert fn_stop(stops, chunks) == O.reference_stop_matcher(stops, chunks)
    for data, flush in repair:
        assert fn_repair(data, flush) == O.reference_utf8_repair(data, flush)
    from g4dense_b200.api import Tokenizer
    J, RJ = Tokenizer(tok_paths["joined"]), O.ReferenceTokenizer(tok_paths["joined"])
    for text, bos in enc[:100]:
        assert J.encode(text, bos) == RJ.encode(text, bos)


def test_engine_chat_template_json_forms(engine_tok):
    """Messages as a JSON string (escapes, extra keys, unicode) or as a list."""
    msgs = '[{"role": "system", "content": " s\\u00e9 \\ud83d\\ude00 "}, {"content": "q\\n", "role": "user", "x": [1, {"y": null}]}]'
    want = ("<bos><|turn>system\nsé 😀<turn|>\n<|turn>user\nq<turn|>\n"
            "<|turn>model\n<|channel>thought\n<channel|>").encode()
    assert engine_tok.chat_template(msgs) == want
    assert engine_tok.chat_template([("system", " sé 😀 "), ("user", "q\n")]) == want
    with pytest.raises(RuntimeError, match="chat messages JSON: unterminated string"):
        engine_tok.chat_template('[{"role": "user", "content": "unterminated}]')
    with pytest.raises(RuntimeError, match="chat messages JSON: expected"):
        engine_tok.chat_template('{"role": "user"}')
    with pytest.raises(RuntimeError, match="system message must come first"):
        engine_tok.chat_template([("user", "a"), ("system", "b")])


def test_engine_tokenizer_errors(built_lib, tmp_path):
    from g4dense_b200.api import Tokenizer
    with pytest.raises(RuntimeError, match="no vocabulary path"):
        Tokenizer("")
    with pytest.raises(RuntimeError, match="Failed to open tokenizer"):
        Tokenizer(tmp_path / "definitely_not_a_real_vocab_file.json")
    (tmp_path / "empty.json").write_bytes(b"")
    with pytest.raises(RuntimeError, match="Empty tokenizer file"):
        Tokenizer(tmp_path / "empty.json")
    (tmp_path / "nomodel.json").write_text('{"added_tokens": []}')
    with pytest.raises(RuntimeError, match='no "model" section'):
        Tokenizer(tmp_path / "nomodel.json")
    (tmp_path / "novocab.json").write_text('{"model": {"merges": []}}')
    with pytest.raises(RuntimeError, match="no model.vocab"):
        Tokenizer(tmp_path / "novocab.json")
    (tmp_path / "emptyvocab.json").write_text('{"model": {"vocab": {}}}')
    with pytest.raises(RuntimeError, match="vocabulary is empty"):
        Tokenizer(tmp_path / "emptyvocab.json")
    (tmp_path / "trunc.json").write_text('{"model": {"vocab": {"a": 0, "b"')
    with pytest.raises(RuntimeError, match="tokenizer.json"):
        Tokenizer(tmp_path / "trunc.json")
    with pytest.raises(RuntimeError, match="architecture"):
        Tokenizer(tmp_path / "trunc.json", arch=7)


def test_engine_bpe_is_not_quadratic(engine_tok, tok_paths):
    """A 200 KB segment with no added tokens: the heap BPE finishes in well under a second where
    a rescan per merge would take minutes. Output equals the reference's on a prefix."""
    rng = np.random.default_rng(1)
    from g4dense_b200.synth_tokenizer import SYLLABLES
    text = " ".join("".join(SYLLABLES[i] for i in rng.integers(0, len(SYLLABLES), 3)) for _ in range(25000)).encode()
    t0 = time.perf_counter()
    ids = engine_tok.encode(text, False)
    dt = time.perf_counter() - t0
    assert engine_tok.decode(ids) == text
    print(f"encode of {len(text)} bytes -> {len(ids)} ids in {dt * 1e3:.1f} ms")
    assert dt < 5.0
    head = text[:3000]
    assert engine_tok.encode(head, False) == TO.Tokenizer(tok_paths["pair"]).encode(head, False)


# ---------------------------------------------------------------- the reference's own test cases

def _mini_vocab(tmp_path):
    """tests/test_tokenizer.cpp:63-84's synthetic vocabulary."""
    p = tmp_path / "test_mini_vocab.json"
    p.write_text(json.dumps({
        "added_tokens": [{"id": 0, "content": "<pad>", "special": True}, {"id": 1, "content": "<eos>", "special": True},
                         {"id": 2, "content": "<bos>", "special": True},
                         {"id": 105, "content": "<start_of_turn>", "special": True},
                         {"id": 106, "content": "<end_of_turn>", "special": True},
                         {"id": 107, "content": "\n", "special": False}],
        "model": {"vocab": {"<pad>": 0, "<eos>": 1, "<bos>": 2, "<start_of_turn>": 105, "<end_of_turn>": 106,
                            "\n": 107, "user": 2364, "model": 4368, "Hi": 10979}, "merges": []}}))
    return p


def _detok_vocab(tmp_path):
    """tests/test_detokenizer.cpp:23-43's vocabulary: Hi 2, ' there' 3, ! 4, <0xNN> at 100 + NN."""
    parts = ['{"added_tokens":[{"id":0,"content":"<pad>","special":true},{"id":1,"content":"<eos>","special":true}],'
             '"model":{"vocab":{"<pad>":0,"<eos>":1,"Hi":2," there":3,"!":4']
    parts += [f',"<0x{b:02X}>":{100 + b}' for b in range(256)]
    parts.append('},"merges":[]}}')
    p = tmp_path / "test_detok_vocab.json"
    p.write_text("".join(parts))
    return p


def test_reference_unit_cases(built_lib, tmp_path):
    from g4dense_b200.api import StopMatcher, Tokenizer
    # tests/test_tokenizer.cpp:63-95: the chat template over a mini vocabulary.
    mini = Tokenizer(_mini_vocab(tmp_path))
    assert mini.chat_template([("user", "Hi")]) == b"<bos><|turn>user\nHi<turn|>\n<|turn>model\n<|channel>thought\n<channel|>"
    # the unresolved names keep their default ids; those present are looked up
    assert mini.special_ids() == {"bos": 2, "eos": 1, "pad": 0, "unk": 3, "end_of_turn": 106, "vocab_size": 10980}
    assert mini.stop_ids() == [1, 106, 50]
    # :97-113: Muse-Glimmer special ids and template.
    muse = Tokenizer(_mini_vocab(tmp_path), arch=1)
    assert muse.special_ids()["bos"] == 200000 and muse.special_ids()["eos"] == 200001
    assert muse.stop_ids() == [200001, 200008]
    assert muse.chat_template([("user", "Hello world")]) == \
        b"<|start|>user\n<|message|>Hello world<|eot|>\n<|start|>assistant\n<|message|>"
    # tests/test_detokenizer.cpp:64-105.
    tok = Tokenizer(_detok_vocab(tmp_path))
    d = tok.detokenizer()
    assert d.push(100 + 0xE2) == b"" and d.push(100 + 0x82) == b"" and d.push(100 + 0xAC) == "€".encode()
    assert d.finish() == b""
    d = tok.detokenizer()
    assert d.push(100 + 0xE2) == b"" and d.finish() == b"\xef\xbf\xbd"
    d = tok.detokenizer()
    assert b"".join([d.push(100 + 0xE2), d.push(100 + 0x82), d.push(100 + 0xAC), d.push(2), d.finish()]) == "€Hi".encode()
    d = tok.detokenizer()
    assert b"".join([d.push(2), d.push(1), d.push(4), d.finish()]) == b"Hi!"
    # :113-147 and tests/test_tokenizer.cpp:115-131: the stop matcher.
    m = StopMatcher([b"<eos>"])
    assert m.push(b"<eos>") == b"" and m.stopped and m.matched == b"<eos>"
    m = StopMatcher([b"<start_of_turn>user"])
    assert m.push(b"<start_of_turn>") == b"" and not m.stopped
    assert m.push(b"user") == b"" and m.stopped and m.matched == b"<start_of_turn>user"
    m = StopMatcher([b"<start_of_turn>model"])
    out = m.push(b"<start_of_turn>")
    assert out == b"" and not m.stopped
    out += m.push(b"user") + m.finish()
    assert not m.stopped and out == b"<start_of_turn>user"
    # :149-167: streaming equals batch decoding on 200 random byte sequences.
    rng = np.random.default_rng(0xD370C0D3)
    for _ in range(200):
        ids = (100 + rng.integers(0, 256, int(rng.integers(1, 65)))).tolist()
        d = tok.detokenizer()
        assert b"".join([d.push(t) for t in ids] + [d.finish()]) == tok.decode(ids, False)


def test_text_prompts_have_clear_greedy_margins(config0, tok_paths):
    """The engine's text-generation tests compare streams exactly; that is meaningful only where
    the oracle's greedy choice is not a near-tie (top-1 minus top-2 logit >= 0.05 everywhere)."""
    from g4dense_b200.synth_tokenizer import RAW_PROMPTS, STOP_PROMPT
    T = TO.Tokenizer(tok_paths["pair"])
    tgt = config0["target_centered"]
    cases = [(T.encode(T.chat_template([("user", STOP_PROMPT)]), False), 48, True)]
    cases += [(T.encode(p.encode(), True), 40, False) for p in RAW_PROMPTS]
    for ids, n, must_stop in cases:
        toks, _ = O.spec_generate(O.RestatedModel(tgt), None, ids, n)
        toks = toks.tolist()
        cut = next((i for i, t in enumerate(toks) if t in T.stop_ids), None)
        assert (cut is not None) == must_stop
        toks = toks if cut is None else toks[:cut + 1]
        assert min(O.greedy_margins(tgt, ids, toks)) >= 0.05
