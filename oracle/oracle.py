"""ctypes bindings for the parity checkers. TEST INFRASTRUCTURE ONLY.

* ``Restated``: oracle/_build/libg4oracle.so, our C restatement (g4d_oracle.c). Built on
  demand with gcc when missing, so it is available on any box.
* ``Reference``: oracle/_ref/libg4ref.so, the reference's own CPU code (built here from the
  read-only reference checkout; the prebuilt .so travels with the tree). ``available()``
  says whether it is present.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import this module.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
RESTATED_SO = HERE / "_build" / "libg4oracle.so"
REF_SO = HERE / "_ref" / "libg4ref.so"

_u32p = ctypes.POINTER(ctypes.c_uint32)
_vp = ctypes.c_void_p


def _ptr(a):
    return a.ctypes.data_as(_vp) if a is not None else None


class Sampling(ctypes.Structure):
    _fields_ = [("temperature", ctypes.c_float), ("top_p", ctypes.c_float), ("top_k", ctypes.c_int),
                ("repetition_penalty", ctypes.c_float), ("has_seed", ctypes.c_int),
                ("seed", ctypes.c_uint64)]

    @classmethod
    def greedy(cls):
        return cls(0.0, 1.0, 0, 1.0, 0, 0)


def build_restated() -> Path:
    """(Re)builds the restatement incrementally with make (gcc is on every box)."""
    subprocess.run(["make", "-s", "-C", str(HERE), "restate"], check=True)
    return RESTATED_SO


def build_reference(ref_root: str | None = None) -> Path | None:
    """Builds oracle/_ref from the reference checkout `ref_root` (default: the REF_ROOT
    environment variable) when that directory exists; returns the .so or None."""
    ref_root = ref_root or os.environ.get("REF_ROOT")
    if ref_root and Path(ref_root).is_dir():
        subprocess.run(["make", "-s", "-C", str(HERE), "ref", f"REF_ROOT={ref_root}"], check=True)
    return REF_SO if REF_SO.exists() else None


_restated = None


def restated_lib():
    global _restated
    if _restated is None:
        lib = ctypes.CDLL(str(build_restated()))
        lib.g4o_last_error.restype = ctypes.c_char_p
        lib.g4o_open.restype = _vp
        lib.g4o_open.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_uint32, ctypes.c_int]
        lib.g4o_close.argtypes = [_vp]
        lib.g4o_info.argtypes = [_vp, _vp]
        lib.g4o_length.argtypes = [_vp]
        lib.g4o_length.restype = ctypes.c_uint32
        lib.g4o_truncate.argtypes = [_vp, ctypes.c_uint32]
        lib.g4o_forward.argtypes = [_vp, ctypes.c_uint32, ctypes.c_uint32, _vp, _vp]
        lib.g4o_int4_gemm.argtypes = [_vp, _vp, _vp, ctypes.c_uint32, ctypes.c_uint32, _vp,
                                      ctypes.c_uint32, _vp]
        lib.g4o_int8_gemv.argtypes = [_vp, _vp, _vp, ctypes.c_uint32, ctypes.c_uint32, _vp, _vp]
        lib.g4o_attn_gate.argtypes = [_vp, _vp, _vp, ctypes.c_uint32]
        lib.g4o_rmsnorm.argtypes = [_vp, _vp, ctypes.c_uint32, ctypes.c_float, _vp]
        lib.g4o_attention.argtypes = [_vp, _vp, _vp] + [ctypes.c_uint32] * 6 + [ctypes.c_float, _vp]
        lib.g4o_round_f16.restype = ctypes.c_float
        lib.g4o_round_f16.argtypes = [ctypes.c_float]
        lib.g4o_round_bf16.restype = ctypes.c_float
        lib.g4o_round_bf16.argtypes = [ctypes.c_float]
        lib.g4o_gelu_tanh.restype = ctypes.c_float
        lib.g4o_gelu_tanh.argtypes = [ctypes.c_float]
        lib.g4o_splitmix64.restype = ctypes.c_uint64
        lib.g4o_splitmix64.argtypes = [ctypes.c_uint64]
        lib.g4o_seed_for.restype = ctypes.c_uint64
        lib.g4o_seed_for.argtypes = [ctypes.POINTER(Sampling), ctypes.c_int]
        lib.g4o_validate_sampling.argtypes = [ctypes.POINTER(Sampling)]
        lib.g4o_sample_token.restype = ctypes.c_uint32
        lib.g4o_sample_token.argtypes = [_vp, ctypes.c_uint32, ctypes.POINTER(Sampling), ctypes.c_uint64]
        lib.g4o_argmax.restype = ctypes.c_uint32
        lib.g4o_argmax.argtypes = [_vp, ctypes.c_uint32]
        lib.g4o_evaluate_verification.argtypes = [_vp, ctypes.c_int, _vp, ctypes.c_int, ctypes.c_uint32,
                                                  ctypes.POINTER(Sampling), ctypes.c_uint64, _vp, _vp, _vp]
        lib.g4o_mt64_seed.argtypes = [_vp, ctypes.c_uint64]
        lib.g4o_mt64_uniform_float.restype = ctypes.c_float
        lib.g4o_mt64_uniform_float.argtypes = [_vp]
        lib.g4o_spec_generate.argtypes = [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                          ctypes.POINTER(Sampling), ctypes.c_double, ctypes.c_int,
                                          ctypes.c_int64, _vp, ctypes.c_int, ctypes.c_double,
                                          ctypes.c_uint64, _vp, _vp, ctypes.c_int, _vp]
        lib.g4o_mtp_open.restype = _vp
        lib.g4o_mtp_open.argtypes = [ctypes.c_char_p]
        lib.g4o_mtp_close.argtypes = [_vp]
        lib.g4o_mtp_info.argtypes = [_vp, _vp]
        lib.g4o_mtp_draft.argtypes = [_vp, _vp, _vp, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                                      ctypes.POINTER(Sampling), _vp, _vp]
        _restated = lib
    return _restated


KV_FP16, KV_BF16, KV_FP32 = 0, 1, 2


class RestatedModel:
    """Our C restatement of CpuReferenceRunner, with a truncatable KV cache."""

    def __init__(self, path, kv_mode=KV_FP16, max_ctx=4096, cache_dequant=True):
        self.lib = restated_lib()
        self.h = self.lib.g4o_open(str(path).encode(), kv_mode, max_ctx, 1 if cache_dequant else 0)
        if not self.h:
            raise RuntimeError(self.lib.g4o_last_error().decode())
        info = np.zeros(12, np.uint32)
        self.lib.g4o_info(self.h, _ptr(info))
        (self.num_layers, self.d_model, self.d_ff, self.q_heads, self.kv_heads, self.head_dim,
         self.vocab, self.window, self.global_head_dim, self.global_kv_heads) = [int(x) for x in info[:10]]
        self.global_mask = int(info[10]) | (int(info[11]) << 32)

    def close(self):
        if self.h:
            self.lib.g4o_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def length(self):
        return int(self.lib.g4o_length(self.h))

    def truncate(self, n):
        self.lib.g4o_truncate(self.h, n)

    def forward(self, token, pos, want_hidden=False):
        logits = np.empty(self.vocab, np.float32)
        hidden = np.empty(self.d_model, np.float32) if want_hidden else None
        if self.lib.g4o_forward(self.h, token, pos, _ptr(logits), _ptr(hidden)):
            raise RuntimeError(self.lib.g4o_last_error().decode())
        return (logits, hidden) if want_hidden else logits


class RestatedMtp:
    """Our C restatement of MtpRunner (src/mtp_runner.cpp) over a RestatedModel target."""

    def __init__(self, path):
        self.lib = restated_lib()
        self.h = self.lib.g4o_mtp_open(str(path).encode())
        if not self.h:
            raise RuntimeError(self.lib.g4o_last_error().decode())
        info = np.zeros(12, np.uint32)
        self.lib.g4o_mtp_info(self.h, _ptr(info))
        self.vocab = int(info[4])

    def close(self):
        if self.h:
            self.lib.g4o_mtp_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def draft(self, target: RestatedModel, hidden, seed_token, context_length, k, sampling: Sampling | None = None):
        """(tokens [k], logits [k][vocab]) drafted from the target's state."""
        sp = sampling or Sampling.greedy()
        toks = np.zeros(k, np.uint32)
        logits = np.zeros((k, self.vocab), np.float32)
        hid = np.ascontiguousarray(hidden, np.float32)
        if self.lib.g4o_mtp_draft(self.h, target.h, _ptr(hid), seed_token, context_length, k, ctypes.byref(sp),
                                  _ptr(toks), _ptr(logits)):
            raise RuntimeError(self.lib.g4o_last_error().decode())
        return toks, logits


def spec_generate(target: RestatedModel, draft: RestatedModel | None, prompt, max_tokens,
                  verify_width=5, sampling: Sampling | None = None, gate_min_accept=0.45,
                  gate_window=24, stop_id=-1, replay_stream=None, mismatch_rate=0.0,
                  mismatch_seed=0):
    """Restated ForwardRunner::generate (src/runner.cpp:2120-2347). Returns
    (tokens, rounds) with rounds = [(drafted, accepted, emitted), ...]."""
    lib = restated_lib()
    sp = sampling or Sampling.greedy()
    prompt = np.ascontiguousarray(prompt, np.uint32)
    out = np.zeros(max_tokens + 16, np.uint32)
    max_rounds = max_tokens + 16
    ri = np.zeros(3 * max_rounds, np.int32)
    nr = ctypes.c_int(0)
    rs = None if replay_stream is None else np.ascontiguousarray(replay_stream, np.uint32)
    n = lib.g4o_spec_generate(target.h, draft.h if draft else None, _ptr(prompt), len(prompt),
                              max_tokens, verify_width, ctypes.byref(sp), gate_min_accept,
                              gate_window, stop_id, _ptr(rs), 0 if rs is None else len(rs),
                              mismatch_rate, mismatch_seed, _ptr(out), _ptr(ri), max_rounds,
                              ctypes.byref(nr))
    if n < 0:
        raise RuntimeError(lib.g4o_last_error().decode())
    return out[:n].copy(), [tuple(int(v) for v in ri[3 * i:3 * i + 3]) for i in range(nr.value)]


def greedy_margins(path, prompt, tokens):
    """Top-1 minus top-2 logit of the target along a given continuation (teacher-forced):
    margins[i] belongs to the distribution that produced tokens[i]."""
    m = RestatedModel(path)
    prompt = [int(t) for t in prompt]
    for p, t in enumerate(prompt[:-1]):
        m.forward(t, p)
    out = []
    prev, pos = prompt[-1], len(prompt) - 1
    for t in tokens:
        s = np.sort(m.forward(prev, pos))[::-1]
        out.append(float(s[0] - s[1]))
        prev, pos = int(t), pos + 1
    m.close()
    return out


def int4_gemm(W, S, B, x):
    """Restated GemmInt4Batch: W u32 [N][K/8], S/B u16 [N][K/64], x f32 [M][K] -> [M][N]."""
    lib = restated_lib()
    W = np.ascontiguousarray(W, np.uint32)
    S = np.ascontiguousarray(S, np.uint16)
    B = np.ascontiguousarray(B, np.uint16)
    x = np.ascontiguousarray(x, np.float32)
    N, K = W.shape[0], W.shape[1] * 8
    M = x.shape[0]
    out = np.empty((M, N), np.float32)
    lib.g4o_int4_gemm(_ptr(W), _ptr(S), _ptr(B), N, K, _ptr(x), M, _ptr(out))
    return out


def int8_gemv(W, S, B, x):
    lib = restated_lib()
    W = np.ascontiguousarray(W, np.uint32)
    N, K = W.shape[0], W.shape[1] * 4
    out = np.empty(N, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    lib.g4o_int8_gemv(_ptr(W), _ptr(np.ascontiguousarray(S, np.uint16)),
                      _ptr(np.ascontiguousarray(B, np.uint16)), N, K, _ptr(x), _ptr(out))
    return out


def attn_gate(ctx, gate):
    lib = restated_lib()
    ctx = np.ascontiguousarray(ctx, np.float32)
    gate = np.ascontiguousarray(gate, np.float32)
    out = np.empty_like(ctx)
    lib.g4o_attn_gate(_ptr(ctx), _ptr(gate), _ptr(out), ctx.size)
    return out


def evaluate_verification(drafts, target_logits, sampling=None, base_seed=0, draft_logits=None):
    lib = restated_lib()
    sp = sampling or Sampling.greedy()
    d = np.ascontiguousarray(drafts, np.uint32)
    tl = np.ascontiguousarray(target_logits, np.float32)
    dl = None if draft_logits is None else np.ascontiguousarray(draft_logits, np.float32)
    out = np.zeros(len(d) + 1, np.uint32)
    na = ctypes.c_uint32(0)
    n = lib.g4o_evaluate_verification(_ptr(d), len(d), _ptr(tl), tl.shape[0], tl.shape[1],
                                      ctypes.byref(sp), base_seed, _ptr(dl), _ptr(out), ctypes.byref(na))
    return out[:n].tolist(), int(na.value)


# ---------------------------------------------------------------- the reference's own code

_ref = None


def reference_available() -> bool:
    return REF_SO.exists()


def reference_lib():
    global _ref
    if _ref is None:
        if not REF_SO.exists():
            raise FileNotFoundError(f"{REF_SO} is not built (make -C oracle ref)")
        lib = ctypes.CDLL(str(REF_SO))
        lib.ref_last_error.restype = ctypes.c_char_p
        lib.ref_open.restype = _vp
        lib.ref_open.argtypes = [ctypes.c_char_p]
        lib.ref_close.argtypes = [_vp]
        lib.ref_vocab.argtypes = [_vp]
        lib.ref_vocab.restype = ctypes.c_uint32
        lib.ref_forward.argtypes = [_vp, ctypes.c_uint32, ctypes.c_uint32, _vp]
        lib.ref_reset.argtypes = [_vp]
        lib.ref_splitmix64.restype = ctypes.c_uint64
        lib.ref_splitmix64.argtypes = [ctypes.c_uint64]
        lib.ref_seed_for.restype = ctypes.c_uint64
        lib.ref_seed_for.argtypes = [ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.c_float,
                                     ctypes.c_int, ctypes.c_uint64, ctypes.c_int]
        lib.ref_sample_token.restype = ctypes.c_uint32
        lib.ref_sample_token.argtypes = [_vp, ctypes.c_uint32, ctypes.c_float, ctypes.c_float, ctypes.c_int,
                                         ctypes.c_float, ctypes.c_int, ctypes.c_uint64, ctypes.c_uint64]
        lib.ref_validate_sampling.argtypes = [ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.c_float]
        lib.ref_evaluate_verification.argtypes = [_vp, ctypes.c_int, _vp, ctypes.c_int, ctypes.c_uint32,
                                                  ctypes.c_float, ctypes.c_float, ctypes.c_int,
                                                  ctypes.c_float, ctypes.c_int, ctypes.c_uint64,
                                                  ctypes.c_uint64, _vp, _vp, _vp]
        lib.ref_spec_generate.argtypes = [ctypes.c_char_p, ctypes.c_char_p, _vp, ctypes.c_int, ctypes.c_int,
                                          ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_int,
                                          ctypes.c_int, ctypes.c_uint64, ctypes.c_double, ctypes.c_int,
                                          ctypes.c_int64, _vp, _vp, ctypes.c_int, _vp]
        sz = ctypes.POINTER(ctypes.c_size_t)
        lib.ref_tok_open.restype = _vp
        lib.ref_tok_open.argtypes = [ctypes.c_char_p, ctypes.c_int]
        lib.ref_tok_close.argtypes = [_vp]
        lib.ref_tok_encode.argtypes = [_vp, ctypes.c_char_p, ctypes.c_size_t, ctypes.c_int, _vp, ctypes.c_int]
        lib.ref_tok_decode.restype = _vp
        lib.ref_tok_decode.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int, sz]
        lib.ref_tok_decode_single.restype = _vp
        lib.ref_tok_decode_single.argtypes = [_vp, ctypes.c_uint32, ctypes.c_int, sz]
        lib.ref_tok_chat_template.restype = ctypes.c_char_p
        lib.ref_tok_chat_template.argtypes = [_vp, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(ctypes.c_char_p),
                                              ctypes.c_int]
        lib.ref_tok_special_ids.argtypes = [_vp, _vp]
        lib.ref_tok_stop_ids.argtypes = [_vp, _vp, ctypes.c_int]
        lib.ref_tok_byte_value.argtypes = [_vp, ctypes.c_uint32, ctypes.POINTER(ctypes.c_uint8)]
        lib.ref_tok_is_special.argtypes = [_vp, ctypes.c_uint32]
        lib.ref_detok_create.restype = _vp
        lib.ref_detok_create.argtypes = [_vp, ctypes.c_int]
        lib.ref_detok_push.restype = _vp
        lib.ref_detok_push.argtypes = [_vp, ctypes.c_uint32, sz]
        lib.ref_detok_finish.restype = _vp
        lib.ref_detok_finish.argtypes = [_vp, sz]
        lib.ref_detok_destroy.argtypes = [_vp]
        lib.ref_stop_create.restype = _vp
        lib.ref_stop_create.argtypes = [ctypes.POINTER(ctypes.c_char_p), ctypes.c_int]
        lib.ref_stop_push.restype = _vp
        lib.ref_stop_push.argtypes = [_vp, ctypes.c_char_p, ctypes.c_size_t, sz]
        lib.ref_stop_finish.restype = _vp
        lib.ref_stop_finish.argtypes = [_vp, sz]
        lib.ref_stop_stopped.argtypes = [_vp, ctypes.POINTER(ctypes.c_char_p)]
        lib.ref_stop_destroy.argtypes = [_vp]
        lib.ref_utf8_repair.restype = _vp
        lib.ref_utf8_repair.argtypes = [ctypes.c_char_p, ctypes.c_size_t, ctypes.c_int, sz, sz]
        _ref = lib
    return _ref


class ReferenceModel:
    """The reference's CpuReferenceRunner (append-only KV)."""

    def __init__(self, path):
        self.lib = reference_lib()
        self.h = self.lib.ref_open(str(path).encode())
        if not self.h:
            raise RuntimeError(self.lib.ref_last_error().decode())
        self.vocab = int(self.lib.ref_vocab(self.h))

    def forward(self, token, pos):
        out = np.empty(self.vocab, np.float32)
        if self.lib.ref_forward(self.h, token, pos, _ptr(out)):
            raise RuntimeError(self.lib.ref_last_error().decode())
        return out

    def reset(self):
        self.lib.ref_reset(self.h)

    def close(self):
        if self.h:
            self.lib.ref_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def reference_spec_generate(target_path, draft_path, prompt, max_tokens, verify_width=5,
                            sampling: Sampling | None = None, gate_min_accept=0.45,
                            gate_window=24, stop_id=-1):
    lib = reference_lib()
    sp = sampling or Sampling.greedy()
    prompt = np.ascontiguousarray(prompt, np.uint32)
    out = np.zeros(max_tokens + 16, np.uint32)
    max_rounds = max_tokens + 16
    ri = np.zeros(3 * max_rounds, np.int32)
    nr = ctypes.c_int(0)
    n = lib.ref_spec_generate(str(target_path).encode(),
                              None if draft_path is None else str(draft_path).encode(),
                              _ptr(prompt), len(prompt), max_tokens, verify_width, sp.temperature,
                              sp.top_p, sp.top_k, sp.has_seed, sp.seed, gate_min_accept, gate_window,
                              stop_id, _ptr(out), _ptr(ri), max_rounds, ctypes.byref(nr))
    if n < 0:
        raise RuntimeError(lib.ref_last_error().decode())
    return out[:n].copy(), [tuple(int(v) for v in ri[3 * i:3 * i + 3]) for i in range(nr.value)]


def reference_evaluate_verification(drafts, target_logits, sampling=None, base_seed=0, draft_logits=None):
    lib = reference_lib()
    sp = sampling or Sampling.greedy()
    d = np.ascontiguousarray(drafts, np.uint32)
    tl = np.ascontiguousarray(target_logits, np.float32)
    dl = None if draft_logits is None else np.ascontiguousarray(draft_logits, np.float32)
    out = np.zeros(len(d) + 1, np.uint32)
    na = ctypes.c_uint32(0)
    n = lib.ref_evaluate_verification(_ptr(d), len(d), _ptr(tl), tl.shape[0], tl.shape[1],
                                      sp.temperature, sp.top_p, sp.top_k, sp.repetition_penalty,
                                      sp.has_seed, sp.seed, base_seed, _ptr(dl), _ptr(out), ctypes.byref(na))
    if n < 0:
        raise RuntimeError(lib.ref_last_error().decode())
    return out[:n].tolist(), int(na.value)


class ReferenceTokenizer:
    """The reference's own Tokenizer / IncrementalDetokenizer / StreamingStopMatcher
    (src/tokenizer.cpp, src/detokenizer.cpp, compiled unmodified into oracle/_ref). Same method
    shapes as g4dense_b200.api.Tokenizer; text in as bytes, out as bytes."""

    def __init__(self, path=None, arch=0):
        self.lib = reference_lib()
        self.h = self.lib.ref_tok_open(None if path is None else str(path).encode(), arch)
        if not self.h:
            raise RuntimeError(self.lib.ref_last_error().decode())

    def _take(self, p, n):
        if not p:
            raise RuntimeError(self.lib.ref_last_error().decode())
        return ctypes.string_at(p, n.value)

    def encode(self, text: bytes, add_bos=True):
        n = self.lib.ref_tok_encode(self.h, text, len(text), 1 if add_bos else 0, None, 0)
        if n < 0:
            raise RuntimeError(self.lib.ref_last_error().decode())
        out = np.zeros(max(n, 1), np.uint32)
        self.lib.ref_tok_encode(self.h, text, len(text), 1 if add_bos else 0, _ptr(out), len(out))
        return out[:n].tolist()

    def decode(self, ids, skip_special=True):
        a = np.ascontiguousarray(ids, np.uint32)
        n = ctypes.c_size_t(0)
        return self._take(self.lib.ref_tok_decode(self.h, _ptr(a), len(a), 1 if skip_special else 0,
                                                  ctypes.byref(n)), n)

    def decode_single(self, tid, skip_special=True):
        n = ctypes.c_size_t(0)
        return self._take(self.lib.ref_tok_decode_single(self.h, tid, 1 if skip_special else 0, ctypes.byref(n)), n)

    def chat_template(self, messages):
        """messages: [(role, content)] as bytes or str."""
        enc = [tuple(x if isinstance(x, bytes) else x.encode() for x in m) for m in messages]
        roles = (ctypes.c_char_p * max(1, len(enc)))(*[m[0] for m in enc])
        contents = (ctypes.c_char_p * max(1, len(enc)))(*[m[1] for m in enc])
        r = self.lib.ref_tok_chat_template(self.h, roles, contents, len(enc))
        if r is None:
            raise RuntimeError(self.lib.ref_last_error().decode())
        return r

    def special_ids(self):
        v = np.zeros(7, np.uint32)
        self.lib.ref_tok_special_ids(self.h, _ptr(v))
        return dict(zip(("bos", "eos", "pad", "unk", "end_of_turn", "vocab_size", "loaded"), v.tolist()))

    def stop_ids(self):
        v = np.zeros(16, np.uint32)
        n = self.lib.ref_tok_stop_ids(self.h, _ptr(v), len(v))
        return v[:n].tolist()

    def byte_value(self, tid):
        b = ctypes.c_uint8(0)
        return b.value if self.lib.ref_tok_byte_value(self.h, tid, ctypes.byref(b)) else None

    def is_special(self, tid):
        return bool(self.lib.ref_tok_is_special(self.h, tid))

    def stream(self, ids, skip_special=True):
        """IncrementalDetokenizer: [push(id) for id in ids] + [finish()]."""
        d = self.lib.ref_detok_create(self.h, 1 if skip_special else 0)
        n = ctypes.c_size_t(0)
        out = [self._take(self.lib.ref_detok_push(d, int(t), ctypes.byref(n)), n) for t in ids]
        out.append(self._take(self.lib.ref_detok_finish(d, ctypes.byref(n)), n))
        self.lib.ref_detok_destroy(d)
        return out

    def __del__(self):
        try:
            if self.h:
                self.lib.ref_tok_close(self.h)
        except Exception:
            pass


def reference_stop_matcher(stops, chunks):
    """StreamingStopMatcher: ([push(c) for c in chunks] + [finish()], stopped, matched)."""
    lib = reference_lib()
    arr = (ctypes.c_char_p * max(1, len(stops)))(*stops)
    m = lib.ref_stop_create(arr, len(stops))
    n = ctypes.c_size_t(0)
    out = [ctypes.string_at(lib.ref_stop_push(m, c, len(c), ctypes.byref(n)), n.value) for c in chunks]
    out.append(ctypes.string_at(lib.ref_stop_finish(m, ctypes.byref(n)), n.value))
    matched = ctypes.c_char_p()
    stopped = bool(lib.ref_stop_stopped(m, ctypes.byref(matched)))
    res = (out, stopped, matched.value or b"")
    lib.ref_stop_destroy(m)
    return res


def reference_utf8_repair(data: bytes, flush_all: bool):
    lib = reference_lib()
    used, n = ctypes.c_size_t(0), ctypes.c_size_t(0)
    p = lib.ref_utf8_repair(data, len(data), 1 if flush_all else 0, ctypes.byref(used), ctypes.byref(n))
    return ctypes.string_at(p, n.value), used.value
