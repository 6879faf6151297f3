"""Writes tests/golden/tokenizer.json: golden vectors for the tokenizer, produced by the
REFERENCE's own Tokenizer / IncrementalDetokenizer / StreamingStopMatcher / utf8_repair
(src/tokenizer.cpp, src/detokenizer.cpp compiled unmodified into oracle/_ref/libg4ref.so) over
the synthetic tokenizer.json of g4dense_b200.synth_tokenizer.

Run from the repository root where the reference checkout exists (oracle/_ref must be built):
    python tests/golden/make_tokenizer_golden.py

Byte strings are stored as hex. The tokenizer files' SHA-256 is stored too, so a test can tell
a changed synthetic vocabulary from a tokenizer bug.
"""
from __future__ import annotations

import hashlib
import json
import sys
import tempfile
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[2]
sys.path[:0] = [str(REPO), str(REPO / "turbo-winfare-dense_b200")]

from g4dense_b200 import synth_tokenizer as S  # noqa: E402
from oracle import oracle as O  # noqa: E402

OUT = Path(__file__).resolve().parent / "tokenizer.json"

# Pieces the random texts are made of: corpus syllables (so merges fire), added tokens and
# near-misses, whitespace runs, non-ASCII characters with and without pieces, and bytes that are
# not valid UTF-8.
FRAGMENTS = ([s.encode() for s in S.SYLLABLES] +
             [b" ", b" ", b" ", b"  ", b"\n", b"\t", b"\r\n", b",", b".", b"!", b"?", b"'", b"-", b"0", b"42"] +
             [c.encode() for c, _ in S.ADDED.values()] +
             [b"<", b"[", b"<|tur", b"<turn", b"<bos", b"[multi", b"<0x41>", b"<unused3>", b"<|", b"|>"] +
             ["é".encode(), "ü".encode(), "中文".encode(), "日本".encode(), "😀".encode(), "€".encode(),
              "ℵ".encode(), "ß".encode(), "©".encode()] +
             [b"\xff", b"\x80", b"\xe2\x82", b"\xc3", b"\xf0\x9f\x98", b"\x00", b"\x7f"])


def random_text(rng, n_frag):
    return b"".join(FRAGMENTS[int(i)] for i in rng.integers(0, len(FRAGMENTS), n_frag))


def make_cases(seed, n_encode=200, n_decode=120, n_stream=100, n_stop=120, n_repair=120):
    rng = np.random.default_rng(seed)
    enc = []
    for i in range(n_encode):
        n = int(rng.integers(0, 40)) if i % 10 else int(rng.integers(60, 200))
        enc.append((random_text(rng, n), bool(rng.integers(0, 2))))
    enc += [(b"", True), (b"", False), (b" ", False), (b"<", False), (b"<bos>", False), (b"<bos>", True)]
    dec = []
    for _ in range(n_decode):
        n = int(rng.integers(0, 60))
        kind = rng.random()
        if kind < 0.4:  # ids below 400: added tokens, byte-fallback pieces and single characters
            ids = rng.integers(0, 400, n)
        elif kind < 0.7:
            ids = rng.integers(0, 4096, n)
        else:  # with out-of-range ids
            ids = rng.integers(0, 5000, n)
        dec.append((ids.tolist(), bool(rng.integers(0, 2))))
    stream = []
    for _ in range(n_stream):
        n = int(rng.integers(0, 50))
        stream.append((rng.integers(0, 420, n).tolist(), bool(rng.integers(0, 2))))
    stop = []
    stop_pool = [b"<eos>", b"<start_of_turn>user", b"\n\n", b"ab", b"a", b"xyzzy", b"", b"the end", b"<turn|>"]
    for _ in range(n_stop):
        stops = [stop_pool[int(i)] for i in rng.integers(0, len(stop_pool), int(rng.integers(0, 4)))]
        chunks = []
        for _ in range(int(rng.integers(0, 12))):
            c = random_text(rng, int(rng.integers(0, 4)))
            if rng.random() < 0.3 and stops:
                s = stops[int(rng.integers(0, len(stops)))]
                cut = int(rng.integers(0, len(s) + 1))
                c = c + s[:cut]
                chunks.append(c)
                c = s[cut:]
            chunks.append(c)
        stop.append((stops, chunks))
    repair = []
    for _ in range(n_repair):
        n = int(rng.integers(0, 24))
        if rng.random() < 0.5:
            data = bytes(rng.integers(0, 256, n).astype(np.uint8))
        else:
            data = random_text(rng, n // 3)
        repair.append((data, bool(rng.integers(0, 2))))
    return enc, dec, stream, stop, repair


CHATS = [
    [("user", "Hi")],
    [("system", "  You are terse.\n"), ("user", "What is 2+2?"), ("assistant", " 4 "), ("user", "\tand 3+3?\r\n")],
    [("user", ""), ("model", "x")],
    [("user", "a"), ("system", "late system")],
    [],
    [("tool", "{\"k\": 1}"), ("user", "café <bos> [multimodal]")],
]


def golden(ref_tok_path, seed):
    R = O.ReferenceTokenizer(ref_tok_path, 0)
    enc, dec, stream, stop, repair = make_cases(seed)
    g = {"encode": [], "decode": [], "decode_single": [], "stream": [], "stop": [], "utf8_repair": [], "chat": []}
    for text, bos in enc:
        g["encode"].append({"text": text.hex(), "add_bos": bos, "ids": R.encode(text, bos)})
    for ids, skip in dec:
        g["decode"].append({"ids": ids, "skip_special": skip, "out": R.decode(ids, skip).hex()})
    h0, h1 = hashlib.sha256(), hashlib.sha256()
    for t in range(4200):
        h0.update(R.decode_single(t, False) + b"\x00")
        h1.update(R.decode_single(t, True) + b"\x00")
    g["decode_single"] = {"ids": 4200, "sha256_keep_special": h0.hexdigest(), "sha256_skip_special": h1.hexdigest(),
                          "samples": {str(t): R.decode_single(t, False).hex() for t in (0, 1, 2, 50, 105, 106, 107, 109,
                                                                                       120, 300, 340, 369, 500, 4095)}}
    g["byte_values"] = {str(t): R.byte_value(t) for t in range(0, 4200) if R.byte_value(t) is not None}
    g["special"] = [t for t in range(4200) if R.is_special(t)]
    for ids, skip in stream:
        g["stream"].append({"ids": ids, "skip_special": skip, "pushes": [p.hex() for p in R.stream(ids, skip)]})
    for stops, chunks in stop:
        outs, stopped, matched = O.reference_stop_matcher(stops, chunks)
        g["stop"].append({"stops": [s.hex() for s in stops], "chunks": [c.hex() for c in chunks],
                          "outs": [o.hex() for o in outs], "stopped": stopped, "matched": matched.hex()})
    for data, flush in repair:
        out, used = O.reference_utf8_repair(data, flush)
        g["utf8_repair"].append({"in": data.hex(), "flush_all": flush, "out": out.hex(), "consumed": used})
    for arch in (0, 1):
        A = O.ReferenceTokenizer(ref_tok_path, arch)
        ids = A.special_ids()
        for msgs in CHATS:
            try:
                out = A.chat_template(msgs).hex()
            except RuntimeError as e:
                out = {"error": str(e)}
            g["chat"].append({"arch": arch, "messages": msgs, "out": out})
        g[f"ids_arch{arch}"] = {**{k: v for k, v in ids.items() if k != "loaded"}, "stop": A.stop_ids()}
    return g


def main():
    if not O.reference_available():
        sys.exit("oracle/_ref/libg4ref.so is not built: make -C oracle ref REF_ROOT=<reference checkout>")
    with tempfile.TemporaryDirectory() as d:
        pair = S.write_synthetic_tokenizer(Path(d) / "pair.json", merges_as_pairs=True)
        joined = S.write_synthetic_tokenizer(Path(d) / "joined.json", merges_as_pairs=False)
        doc = {
            "generator": "tests/golden/make_tokenizer_golden.py",
            "tokenizer": {"vocab_size": 4096, "seed": 0, "n_merges": 600},
            "sha256": {"pair": hashlib.sha256(pair.read_bytes()).hexdigest(),
                       "joined": hashlib.sha256(joined.read_bytes()).hexdigest()},
            "pair": golden(pair, seed=11),
            # the "left right" merge format must give the same ids on the same texts
            "joined_encode": joined_encode(joined),
        }
    OUT.write_text(json.dumps(doc, separators=(",", ":")) + "\n")
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


def joined_encode(joined_path):
    R = O.ReferenceTokenizer(joined_path)
    enc = make_cases(seed=12, n_encode=60, n_decode=0, n_stream=0, n_stop=0, n_repair=0)[0]
    return [{"text": t.hex(), "add_bos": b, "ids": R.encode(t, b)} for t, b in enc]


if __name__ == "__main__":
    main()
