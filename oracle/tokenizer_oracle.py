"""CPU restatement of the reference tokenizer, detokenizer and stop matcher.

TEST INFRASTRUCTURE ONLY: tests/ use it as a checker of the engine's tokenizer; nothing in the
product imports it. Every string is handled as UTF-8 bytes, as the reference's std::string is.

It follows, function by function:
  * load:           Tokenizer::parse_tokenizer_json (src/tokenizer.cpp:204-378) -- added_tokens
                    (content, id, special), model.vocab (id -> piece, piece -> id, <0xNN> byte
                    pieces), model.merges in both formats ("a b" and ["a", "b"]; a string
                    without a space takes no rank; a repeated pair keeps its first rank), special
                    ids resolved by name (:349-369), added tokens sorted longest first (:371-376);
  * set_arch:       Tokenizer::set_architecture (src/tokenizer.cpp:380-409);
  * encode:         Tokenizer::encode (src/tokenizer.cpp:472-520) and bpe_segment (:433-470),
                    the literal O(n^2) rescan: merge the lowest-ranked adjacent pair (the
                    leftmost of equal ranks) until none is in the table;
  * decode_single:  src/tokenizer.cpp:526-543; byte_value: is_byte_fallback (:546-561);
  * utf8_repair:    src/tokenizer.cpp:563-598; decode: :600-632;
  * chat_template:  Tokenizer::apply_chat_template (src/tokenizer.cpp:638-672);
  * Detokenizer:    IncrementalDetokenizer (src/detokenizer.cpp:7-40);
  * StopMatcher:    StreamingStopMatcher (src/detokenizer.cpp:44-101).
Parity pin: tests/test_tokenizer.py checks it against golden vectors that the reference's own
compiled tokenizer produced (tests/golden/tokenizer.json, made by
tests/golden/make_tokenizer_golden.py) and against the reference's unit-test cases.
"""
from __future__ import annotations

import json

SPACE = "▁".encode()
REPLACEMENT = b"\xef\xbf\xbd"
GEMMA4, MUSE_GLIMMER = 0, 1


def _byte_piece(p: bytes):
    if len(p) != 6 or not p.startswith(b"<0x") or p[5:6] != b">":
        return None
    try:
        return int(p[3:5].decode("ascii"), 16) if all(c in b"0123456789abcdefABCDEF" for c in p[3:5]) else None
    except UnicodeDecodeError:
        return None


def _char_len(b: int) -> int:
    if b & 0xF8 == 0xF0:
        return 4
    if b & 0xF0 == 0xE0:
        return 3
    if b & 0xE0 == 0xC0:
        return 2
    return 1


def utf8_repair(data: bytes, flush_all: bool):
    """-> (repaired bytes, bytes of `data` consumed)."""
    out = bytearray()
    i = 0
    while i < len(data):
        c = data[i]
        need = 1 if c < 0x80 else 2 if c & 0xE0 == 0xC0 else 3 if c & 0xF0 == 0xE0 else 4 if c & 0xF8 == 0xF0 else 0
        if need == 0:
            out += REPLACEMENT
            i += 1
            continue
        if i + need > len(data):
            if not flush_all:
                break
            out += REPLACEMENT
            i = len(data)
            break
        out += data[i:i + need]
        i += need
    return bytes(out), i


class Tokenizer:
    def __init__(self, path=None, arch=GEMMA4):
        self.arch = GEMMA4
        self.bos, self.eos, self.pad, self.unk = 2, 1, 0, 3
        self.turn, self.end_of_turn, self.tool_response = 105, 106, 50
        self.vocab_size = 262144
        self.loaded = False
        self.stop_ids = [1, 106, 50]
        self.pieces: list[bytes] = []
        self.ids: dict[bytes, int] = {}
        self.byte_ids: dict[int, int] = {}
        self.ranks: dict[tuple[bytes, bytes], int] = {}
        self.added: list[tuple[bytes, int]] = []
        self.special: list[bool] = []
        if path is not None:
            self.load(path)
        self.set_arch(arch)

    def load(self, path):
        doc = json.loads(open(path, "rb").read().decode("utf-8"))
        for e in doc.get("added_tokens", []):
            content = e.get("content", "").encode()
            tid = int(e.get("id", 0))
            if content:
                self.added.append((content, tid))
                if tid >= len(self.special):
                    self.special += [False] * (tid + 1 - len(self.special))
                self.special[tid] = e.get("special") is True
        if "model" not in doc:
            raise ValueError('tokenizer.json: no "model" section')
        model = doc["model"]
        if "vocab" not in model:
            raise ValueError("tokenizer.json: no model.vocab")
        for piece, tid in model["vocab"].items():
            p = piece.encode()
            if tid >= len(self.pieces):
                self.pieces += [b""] * (tid + 1 - len(self.pieces))
            self.pieces[tid] = p
            self.ids[p] = tid
            b = _byte_piece(p)
            if b is not None:
                self.byte_ids[b] = tid
        rank = 0
        for m in model.get("merges", []):
            if isinstance(m, list):
                left, right = m[0].encode(), m[1].encode()
            else:
                if " " not in m:
                    continue
                left, right = (x.encode() for x in m.split(" ", 1))
            self.ranks.setdefault((left, right), rank)
            rank += 1
        if not self.pieces or not self.ids:
            raise ValueError("tokenizer.json: vocabulary is empty")
        self.vocab_size = len(self.pieces)
        self.special += [False] * (len(self.pieces) - len(self.special))
        self._resolve()
        self.added.sort(key=lambda a: (-len(a[0]), a[0]))
        self.loaded = True

    def _find(self, name, default):
        return self.ids.get(name.encode(), default)

    def _resolve(self):
        if self.arch == MUSE_GLIMMER:
            self.bos, self.eos = 200000, 200001
            self.bos = self._find("<|begin_of_text|>", self.bos)
            self.bos = self._find("<|start|>", self.bos)
            self.eos = self._find("<|end_of_text|>", self.eos)
            self.stop_ids = [self.eos, self._find("<|eot|>", 200008)]
        else:
            self.bos = self._find("<bos>", self.bos)
            self.eos = self._find("<eos>", self.eos)
            self.pad = self._find("<pad>", self.pad)
            self.unk = self._find("<unk>", self.unk)
            self.turn = self._find("<|turn>", self.turn)
            self.end_of_turn = self._find("<turn|>", self.end_of_turn)
            self.tool_response = self._find("<|tool_response>", self.tool_response)
            self.stop_ids = [self.eos, self.end_of_turn, self.tool_response]

    def set_arch(self, arch):
        self.arch = arch
        if arch == MUSE_GLIMMER:
            self.vocab_size = len(self.pieces) if self.pieces else 202048
        else:
            self.bos, self.eos = 2, 1
            self.vocab_size = len(self.pieces) if self.pieces else 262144
        self._resolve()

    def _bpe(self, text: bytes, out: list):
        if not text:
            return
        syms = []
        i = 0
        while i < len(text):
            n = min(_char_len(text[i]), len(text) - i)
            syms.append(text[i:i + n])
            i += n
        while True:
            best, at = None, -1
            for j in range(len(syms) - 1):
                r = self.ranks.get((syms[j], syms[j + 1]))
                if r is not None and (best is None or r < best):
                    best, at = r, j
            if at < 0:
                break
            syms[at:at + 2] = [syms[at] + syms[at + 1]]
        for s in syms:
            if s in self.ids:
                out.append(self.ids[s])
            else:
                out.extend(self.byte_ids.get(b, self.unk) for b in s)

    def encode(self, text: bytes, add_bos=True):
        if not self.loaded:
            raise ValueError("Tokenizer::encode called before a vocabulary was loaded")
        out = [self.bos] if add_bos else []
        pending = bytearray()
        i = 0
        while i < len(text):
            hit = False
            if text[i:i + 1] in (b"<", b"["):
                for content, tid in self.added:
                    if text.startswith(content, i):
                        self._bpe(bytes(pending).replace(b" ", SPACE), out)
                        pending.clear()
                        out.append(tid)
                        i += len(content)
                        hit = True
                        break
            if not hit:
                pending.append(text[i])
                i += 1
        self._bpe(bytes(pending).replace(b" ", SPACE), out)
        return out

    def is_special(self, tid):
        return tid < len(self.special) and self.special[tid]

    def byte_value(self, tid):
        return _byte_piece(self.pieces[tid]) if tid < len(self.pieces) else None

    def decode_single(self, tid, skip_special=True) -> bytes:
        if tid >= len(self.pieces) or (skip_special and self.is_special(tid)):
            return b""
        return self.pieces[tid].replace(SPACE, b" ")

    def decode(self, ids, skip_special=True) -> bytes:
        if not self.loaded:
            raise ValueError("Tokenizer::decode called before a vocabulary was loaded")
        out, run = bytearray(), bytearray()
        for t in ids:
            if t >= len(self.pieces):
                continue
            b = self.byte_value(t)
            if b is not None:
                run.append(b)
                continue
            if run:
                out += utf8_repair(bytes(run), True)[0]
                run.clear()
            out += self.decode_single(t, skip_special)
        if run:
            out += utf8_repair(bytes(run), True)[0]
        return bytes(out)

    def chat_template(self, messages) -> bytes:
        """messages: [(role, content)] as str or bytes."""
        def b(x):
            return x if isinstance(x, bytes) else x.encode()

        def trim(c):
            return c.strip(b" \t\r\n")
        out = bytearray()
        if self.arch == MUSE_GLIMMER:
            for role, content in messages:
                r = b"assistant" if b(role) == b"model" else b(role)
                out += b"<|start|>" + r + b"\n<|message|>" + trim(b(content)) + b"<|eot|>\n"
            return bytes(out) + b"<|start|>assistant\n<|message|>"
        out += b"<bos>"
        for i, (role, content) in enumerate(messages):
            if b(role) == b"system" and i != 0:
                raise ValueError("chat template: a system message must come first")
            r = b"model" if b(role) == b"assistant" else b(role)
            out += b"<|turn>" + r + b"\n" + trim(b(content)) + b"<turn|>\n"
        return bytes(out) + b"<|turn>model\n<|channel>thought\n<channel|>"


class Detokenizer:
    def __init__(self, tok: Tokenizer, skip_special=True):
        self.t, self.skip, self.pending = tok, skip_special, b""

    def _drain(self, flush_all):
        out, used = utf8_repair(self.pending, flush_all)
        self.pending = self.pending[used:]
        return out

    def push(self, tid) -> bytes:
        b = self.t.byte_value(tid)
        if b is not None:
            self.pending += bytes([b])
            return self._drain(False)
        if self.skip and self.t.is_special(tid):
            return self._drain(True)
        out = self._drain(True)
        self.pending += self.t.decode_single(tid, self.skip)
        return out + self._drain(False)

    def finish(self) -> bytes:
        return self._drain(True)


class StopMatcher:
    def __init__(self, stops):
        self.stops = [s for s in stops if s]
        self.longest = max((len(s) for s in self.stops), default=0)
        self.buf, self.matched, self.stopped = b"", b"", False

    def push(self, text: bytes) -> bytes:
        if self.stopped:
            return b""
        if not self.stops:
            return text
        self.buf += text
        at, hit = None, None
        for s in self.stops:
            p = self.buf.find(s)
            if p >= 0 and (at is None or p < at):
                at, hit = p, s
        if hit is not None:
            self.stopped, self.matched = True, hit
            out, self.buf = self.buf[:at], b""
            return out
        hold = 0
        for n in range(min(self.longest - 1 if self.longest else 0, len(self.buf)), 0, -1):
            tail = self.buf[len(self.buf) - n:]
            if any(len(s) > n and s[:n] == tail for s in self.stops):
                hold = n
                break
        out, self.buf = self.buf[:len(self.buf) - hold], self.buf[len(self.buf) - hold:]
        return out

    def finish(self) -> bytes:
        if self.stopped:
            return b""
        out, self.buf = self.buf, b""
        return out
