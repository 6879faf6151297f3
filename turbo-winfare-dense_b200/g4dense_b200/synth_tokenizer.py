"""Synthetic Gemma-4-style ``tokenizer.json`` for tests (the real 262,144-piece file is not
available here).

The file has the three sections the engine's tokenizer reads (Hugging Face layout):
``added_tokens`` (the Gemma-4 special tokens at their real ids -- <pad> 0, <eos> 1, <bos> 2,
<unk> 3, <|tool_response> 50, <|turn> 105, <turn|> 106 -- plus a few more, some starting with
'[' and one not marked special), ``model.vocab`` (the added tokens, 256 byte-fallback pieces
``<0xNN>``, single characters, the pieces BPE merges produce, and ``<unusedN>`` filler up to
``vocab_size``) and ``model.merges``. Merges are learned from a seeded synthetic corpus by plain
BPE training (the most frequent adjacent pair first, ties broken by the pair's text), with
spaces written as U+2581 as the Gemma normalizer does. Characters outside the base alphabet
(emoji, most CJK) have no piece, so they exercise byte fallback.

Everything is a pure function of (vocab_size, seed, n_merges, merges_as_pairs).
"""
from __future__ import annotations

import json
from collections import Counter
from pathlib import Path

import numpy as np

SPACE = "▁"

# id -> (content, special)
ADDED = {
    0: ("<pad>", True), 1: ("<eos>", True), 2: ("<bos>", True), 3: ("<unk>", True), 4: ("<mask>", True),
    46: ("<|tool>", True), 47: ("<tool|>", True), 48: ("<|tool_call>", True), 49: ("<tool_call|>", True),
    50: ("<|tool_response>", True), 51: ("<tool_response|>", True),
    100: ("<|channel>", True), 101: ("<channel|>", True), 105: ("<|turn>", True), 106: ("<turn|>", True),
    107: ("[multimodal]", True), 108: ("<start_of_image>", True), 109: ("[@BOS@]", False),
    110: ("<|image|>", True),
}

BASE_CHARS = ([chr(c) for c in range(33, 127)] + [SPACE, "\n", "\t"] +
              list("éèüñßçàö中文日©"))

SYLLABLES = ["ka", "to", "ri", "en", "the", "ing", "ion", "ar", "qu", "st", "pre", "ex", "ab", "or", "us",
             "ma", "ne", "lo", "vi", "é", "ü", "ña", "ch", "sh", "er", "al", "in", "co", "de",
             "中", "文", "ly", "ed", "un", "re", "'s", "1", "2", "0", "9"]


# Text prompts for the engine's text entry points on BASELINE config 0's zero-mean target (seed 0)
# with this tokenizer: along each greedy continuation the oracle's top-1 minus top-2 logit stays
# at or above 0.05, so the engine's stream must equal the oracle's token for token.
# STOP_PROMPT, wrapped in the chat template, reaches a stop id at index 33 of the stream;
# RAW_PROMPTS are encoded as given (<bos> first; 17 and 22 ids, so tensor-core prefill) and hold
# added tokens and byte-fallback characters.
STOP_PROMPT = "stin évi chch"
RAW_PROMPTS = ("thequexst 🎉中totheneñalyshorarre1", "ex [multimodal]ñaé2ne🎉éing中😀edé[multimodal]sh")


def _corpus(rng: np.random.Generator, n_words: int):
    w = 1.0 / np.arange(1, len(SYLLABLES) + 1) ** 0.8
    w /= w.sum()
    words = Counter()
    for _ in range(n_words):
        k = int(rng.integers(1, 5))
        word = "".join(SYLLABLES[i] for i in rng.choice(len(SYLLABLES), size=k, p=w))
        if rng.random() < 0.2:
            word = word.capitalize()
        if rng.random() < 0.1:
            word += ",.!?"[int(rng.integers(0, 4))]
        words[SPACE + word] += 1
    return words


def _train(words: Counter, n_merges: int):
    seqs = {w: list(w) for w in words}
    merges = []
    for _ in range(n_merges):
        pairs = Counter()
        for w, syms in seqs.items():
            c = words[w]
            for a, b in zip(syms, syms[1:]):
                pairs[(a, b)] += c
        if not pairs:
            break
        best = min(pairs.items(), key=lambda kv: (-kv[1], kv[0]))
        if best[1] < 2:
            break
        a, b = best[0]
        merges.append((a, b))
        for w, syms in seqs.items():
            i, out = 0, []
            while i < len(syms):
                if i + 1 < len(syms) and syms[i] == a and syms[i + 1] == b:
                    out.append(a + b)
                    i += 2
                else:
                    out.append(syms[i])
                    i += 1
            seqs[w] = out
    return merges


def build_tokenizer_json(vocab_size: int = 4096, seed: int = 0, n_merges: int = 600,
                         merges_as_pairs: bool = True) -> str:
    rng = np.random.default_rng(seed)
    merges = _train(_corpus(rng, 3000), n_merges)
    pieces: dict[int, str] = {i: c for i, (c, _) in ADDED.items()}
    seen = set(pieces.values())
    nxt = 0

    def place(p: str):
        nonlocal nxt
        if p in seen:
            return
        while nxt in pieces:
            nxt += 1
        if nxt >= vocab_size:
            raise ValueError("vocab_size too small for the synthetic vocabulary")
        pieces[nxt] = p
        seen.add(p)

    for b in range(256):
        place(f"<0x{b:02X}>")
    for c in BASE_CHARS:
        place(c)
    for a, b in merges:
        place(a + b)
    k = 0
    while len(pieces) < vocab_size:
        place(f"<unused{k}>")
        k += 1
    doc = {
        "version": "1.0",
        "truncation": None,
        "padding": None,
        "added_tokens": [{"id": i, "content": c, "single_word": False, "lstrip": False, "rstrip": False,
                          "normalized": False, "special": s} for i, (c, s) in sorted(ADDED.items())],
        "normalizer": {"type": "Replace", "pattern": {"String": " "}, "content": SPACE},
        "pre_tokenizer": None,
        "model": {
            "type": "BPE",
            "dropout": None,
            "unk_token": "<unk>",
            "byte_fallback": True,
            "vocab": {pieces[i]: i for i in sorted(pieces)},
            "merges": [[a, b] for a, b in merges] if merges_as_pairs else [f"{a} {b}" for a, b in merges],
        },
    }
    return json.dumps(doc, ensure_ascii=False, indent=1)


def write_synthetic_tokenizer(path, vocab_size: int = 4096, seed: int = 0, n_merges: int = 600,
                              merges_as_pairs: bool = True) -> Path:
    path = Path(path)
    path.write_text(build_tokenizer_json(vocab_size, seed, n_merges, merges_as_pairs), encoding="utf-8")
    return path
