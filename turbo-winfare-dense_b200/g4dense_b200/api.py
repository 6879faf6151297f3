"""ctypes bindings of libg4dense_b200.so (include/g4dense/c_api.h, include/g4dense_b200_ops.h).

There is no fallback: if the library is missing, or CUDA is unavailable when a GPU entry
point is called, the call fails loudly.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libg4dense_b200.so"
_vp = ctypes.c_void_p
_lib = None


def lib():
    """Loads the native library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FileNotFoundError(f"{LIB_PATH} is missing: run g4dense_b200.build.build() first")
        L = ctypes.CDLL(str(LIB_PATH))
        L.g4b_last_error.restype = ctypes.c_char_p
        L.g4b_qmat_create.argtypes = [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, _vp, ctypes.POINTER(_vp)]
        L.g4b_qmat_destroy.argtypes = [_vp]
        L.g4b_qmat_gemm.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_int, _vp]
        L.g4b_qmat_prepare_input.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp]
        L.g4b_qmat_run.argtypes = [_vp, ctypes.c_int, _vp, ctypes.c_int, _vp]
        L.g4b_qmat_info.argtypes = [_vp, _vp]
        L.g4b_qmat_run_partial.argtypes = [_vp, ctypes.c_int, _vp]
        L.g4b_qmat_run_noalloc.argtypes = [_vp, ctypes.c_int, _vp, ctypes.c_int, _vp]
        L.g4b_gemv_int8.argtypes = [_vp, _vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, _vp]
        L.g4b_attn_gate.argtypes = [_vp, _vp, _vp] + [ctypes.c_int] * 5 + [_vp]
        L.g4b_qmat_check_error.argtypes = [_vp]
        _bind_engine(L)
        _lib = L
    return _lib


class EngineConfig(ctypes.Structure):
    """G4DenseEngineConfig (include/g4dense/c_api.h)."""
    _fields_ = [("container_path", ctypes.c_char_p), ("synthetic_preset", ctypes.c_char_p),
                ("synthetic_seed", ctypes.c_ulonglong), ("synthetic_centered", ctypes.c_int),
                ("draft_path", ctypes.c_char_p), ("draft_preset", ctypes.c_char_p),
                ("draft_seed", ctypes.c_ulonglong), ("draft_k", ctypes.c_int), ("max_context", ctypes.c_int),
                ("kv_bf16", ctypes.c_int), ("tp_rank", ctypes.c_int), ("tp_size", ctypes.c_int),
                ("nccl_unique_id", ctypes.c_void_p), ("device", ctypes.c_int),
                ("gate_min_accept", ctypes.c_double), ("gate_window", ctypes.c_int),
                ("tokenizer_path", ctypes.c_char_p)]


TOKEN_CB = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_uint, ctypes.c_char_p)


def _bind_engine(L):
    """Binds the engine-level C API (include/g4dense/c_api.h)."""
    L.g4dense_engine_last_error.restype = ctypes.c_char_p
    L.g4dense_engine_create.restype = _vp
    L.g4dense_engine_create.argtypes = [ctypes.c_char_p]
    L.g4dense_engine_create_ex.restype = _vp
    L.g4dense_engine_create_ex.argtypes = [ctypes.POINTER(EngineConfig)]
    L.g4dense_config_default.argtypes = [ctypes.POINTER(EngineConfig)]
    L.g4dense_engine_destroy.argtypes = [_vp]
    L.g4dense_engine_get_telemetry.restype = ctypes.c_char_p
    L.g4dense_engine_get_telemetry.argtypes = [_vp]
    L.g4dense_options_default.argtypes = [_vp]
    L.g4dense_engine_generate.restype = ctypes.c_char_p
    L.g4dense_engine_generate.argtypes = [_vp, ctypes.c_char_p, ctypes.c_int]
    L.g4dense_engine_generate_ex.restype = ctypes.c_char_p
    L.g4dense_engine_generate_ex.argtypes = [_vp, ctypes.c_char_p, _vp, TOKEN_CB, _vp]
    L.g4dense_engine_generate_text.restype = ctypes.c_char_p
    L.g4dense_engine_generate_text.argtypes = [_vp, ctypes.c_char_p, ctypes.c_int, _vp, TOKEN_CB, _vp]
    L.g4dense_engine_generate_tokens.restype = ctypes.c_char_p
    L.g4dense_engine_generate_tokens.argtypes = [_vp, _vp, ctypes.c_int, _vp, TOKEN_CB, _vp]
    L.g4dense_engine_last_tokens.argtypes = [_vp, _vp, ctypes.c_int]
    L.g4dense_engine_last_rounds.argtypes = [_vp, _vp, ctypes.c_int]
    L.g4dense_engine_forward_batch.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_int]
    L.g4dense_engine_set_decode_options.argtypes = [_vp, ctypes.c_longlong, ctypes.c_int, _vp, ctypes.c_int,
                                                    ctypes.c_double, ctypes.c_ulonglong]
    L.g4dense_engine_set_device_sampling.argtypes = [_vp, ctypes.c_int]
    L.g4dense_engine_mtp_draft.argtypes = [_vp, ctypes.c_uint, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp, _vp]
    L.g4dense_engine_draft_steps.argtypes = [_vp, ctypes.c_uint, ctypes.c_int, ctypes.c_int, _vp, _vp]
    L.g4b_sample_workspace.restype = ctypes.c_size_t
    L.g4b_sample_token.argtypes = [_vp, ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_int,
                                   ctypes.c_uint64, _vp, _vp, _vp]
    L.g4dense_engine_last_stop_reason.argtypes = [_vp]
    L.g4dense_engine_switch_tier.argtypes = [_vp, ctypes.c_int]
    L.g4dense_engine_stop.argtypes = [_vp]
    L.g4dense_nccl_unique_id.argtypes = [_vp]
    L.g4dense_engine_last_stats.argtypes = [_vp, _vp, ctypes.c_int]
    L.g4dense_engine_set_gate.argtypes = [_vp, ctypes.c_double, ctypes.c_int]
    L.g4dense_engine_time_pass.restype = ctypes.c_double
    L.g4dense_engine_time_pass.argtypes = [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    _sz = ctypes.POINTER(ctypes.c_size_t)
    L.g4dense_tokenizer_open.restype = _vp
    L.g4dense_tokenizer_open.argtypes = [ctypes.c_char_p, ctypes.c_int]
    L.g4dense_engine_tokenizer.restype = _vp
    L.g4dense_engine_tokenizer.argtypes = [_vp]
    L.g4dense_tokenizer_destroy.argtypes = [_vp]
    L.g4dense_tokenizer_encode.argtypes = [_vp, ctypes.c_char_p, ctypes.c_size_t, ctypes.c_int, _vp, ctypes.c_int]
    L.g4dense_tokenizer_decode.restype = _vp
    L.g4dense_tokenizer_decode.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int, _sz]
    L.g4dense_tokenizer_decode_single.restype = _vp
    L.g4dense_tokenizer_decode_single.argtypes = [_vp, ctypes.c_uint, ctypes.c_int, _sz]
    L.g4dense_tokenizer_chat_template.restype = ctypes.c_char_p
    L.g4dense_tokenizer_chat_template.argtypes = [_vp, ctypes.c_char_p]
    L.g4dense_tokenizer_special_ids.argtypes = [_vp, _vp]
    L.g4dense_tokenizer_stop_ids.argtypes = [_vp, _vp, ctypes.c_int]
    L.g4dense_tokenizer_byte_value.argtypes = [_vp, ctypes.c_uint, ctypes.POINTER(ctypes.c_ubyte)]
    L.g4dense_tokenizer_is_special.argtypes = [_vp, ctypes.c_uint]
    L.g4dense_detokenizer_create.restype = _vp
    L.g4dense_detokenizer_create.argtypes = [_vp, ctypes.c_int]
    L.g4dense_detokenizer_push.restype = _vp
    L.g4dense_detokenizer_push.argtypes = [_vp, ctypes.c_uint, _sz]
    L.g4dense_detokenizer_finish.restype = _vp
    L.g4dense_detokenizer_finish.argtypes = [_vp, _sz]
    L.g4dense_detokenizer_destroy.argtypes = [_vp]
    L.g4dense_stop_matcher_create.restype = _vp
    L.g4dense_stop_matcher_create.argtypes = [ctypes.POINTER(ctypes.c_char_p), ctypes.c_int]
    L.g4dense_stop_matcher_push.restype = _vp
    L.g4dense_stop_matcher_push.argtypes = [_vp, ctypes.c_char_p, ctypes.c_size_t, _sz]
    L.g4dense_stop_matcher_finish.restype = _vp
    L.g4dense_stop_matcher_finish.argtypes = [_vp, _sz]
    L.g4dense_stop_matcher_stopped.argtypes = [_vp, ctypes.POINTER(ctypes.c_char_p)]
    L.g4dense_stop_matcher_destroy.argtypes = [_vp]
    L.g4dense_utf8_repair.restype = _vp
    L.g4dense_utf8_repair.argtypes = [ctypes.c_char_p, ctypes.c_size_t, ctypes.c_int, _sz, _sz]
    L.g4dense_container_validate.argtypes = [ctypes.c_char_p]
    L.g4dense_engine_profile_gemms.restype = ctypes.c_double
    L.g4dense_engine_profile_gemms.argtypes = [_vp, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_ulonglong),
                                               ctypes.POINTER(ctypes.c_int)]


def _check(rc, what):
    if rc != 0:
        raise RuntimeError(f"{what} failed ({rc}): {lib().g4b_last_error().decode()}")


def _dptr(t):
    """Device pointer of a torch CUDA tensor."""
    return ctypes.c_void_p(t.data_ptr())


def _stream(stream):
    return ctypes.c_void_p(stream.cuda_stream if stream is not None else 0)


def gemv_int8(W, S, B, x, out, stream=None):
    """out[r] = sum_k (W[r][k] * s + b) * x[k]: W uint8 [rows][K], S/B bf16 bits [rows][K/64],
    x fp32 [K], out fp32 [rows] (torch CUDA tensors)."""
    _check(lib().g4b_gemv_int8(_dptr(W), _dptr(S), _dptr(B), _dptr(x), _dptr(out), W.shape[0], W.shape[1],
                               _stream(stream)), "g4b_gemv_int8")


def attn_gate(ctx, gate, out, stream=None):
    """out = ctx * sigmoid(gate) over [batch][n] fp32 torch CUDA tensors (row strides honoured)."""
    _check(lib().g4b_attn_gate(_dptr(ctx), _dptr(gate), _dptr(out), ctx.shape[1], ctx.shape[0], ctx.stride(0),
                               gate.stride(0), out.stride(0), _stream(stream)), "g4b_attn_gate")


def sample_workspace_bytes():
    return int(lib().g4b_sample_workspace())


def sample_token(logits, temperature, top_p, top_k, seed, workspace, out, stream=None):
    """Draws a token from the fp32 logits row (torch CUDA tensor) into out (uint32/int32 CUDA
    tensor of one element) as the reference's sample_token does; workspace is a CUDA byte tensor
    of sample_workspace_bytes()."""
    _check(lib().g4b_sample_token(_dptr(logits), logits.numel(), temperature, top_p, top_k, seed & (2**64 - 1),
                                  _dptr(workspace), _dptr(out), _stream(stream)), "g4b_sample_token")


class QMat:
    """A prepared INT4 G64 matrix on the device (g4b_qmat)."""

    def __init__(self, W, S, B, stream=None):
        """W, S, B: torch CUDA tensors in container layout (int32/uint32 [N][K/8],
        int16/uint16 [N][K/64] x2)."""
        self.N = W.shape[0]
        self.K = W.shape[1] * 8
        h = ctypes.c_void_p()
        _check(lib().g4b_qmat_create(_dptr(W), _dptr(S), _dptr(B), self.N, self.K, _stream(stream),
                                     ctypes.byref(h)), "g4b_qmat_create")
        self.h = h

    def gemm(self, x, out, stream=None):
        _check(lib().g4b_qmat_gemm(self.h, _dptr(x), x.shape[1], x.shape[0], _dptr(out), out.shape[1],
                                   _stream(stream)), "g4b_qmat_gemm")

    def prepare(self, x, stream=None):
        _check(lib().g4b_qmat_prepare_input(self.h, _dptr(x), x.shape[1], x.shape[0], _stream(stream)),
               "g4b_qmat_prepare_input")

    def run(self, M, out, stream=None):
        _check(lib().g4b_qmat_run(self.h, M, _dptr(out), out.shape[1], _stream(stream)), "g4b_qmat_run")

    def run_noalloc(self, M, out, stream=None):
        """g4b_qmat_run with the library's static split-K scratch (allocates nothing)."""
        _check(lib().g4b_qmat_run_noalloc(self.h, M, _dptr(out), out.shape[1], _stream(stream)),
               "g4b_qmat_run_noalloc")

    def run_partial(self, M, stream=None):
        _check(lib().g4b_qmat_run_partial(self.h, M, _stream(stream)), "g4b_qmat_run_partial")

    def check_error(self):
        _check(lib().g4b_qmat_check_error(self.h), "g4b_qmat_check_error")

    def info(self):
        o = np.zeros(4, np.int32)
        _check(lib().g4b_qmat_info(self.h, o.ctypes.data_as(_vp)), "g4b_qmat_info")
        return {"N": int(o[0]), "K": int(o[1]), "grid_m5": int(o[2]), "max_slots": int(o[3])}

    def close(self):
        if getattr(self, "h", None):
            lib().g4b_qmat_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class GenOptions(ctypes.Structure):
    """G4DenseGenerationOptions (include/g4dense/c_api.h:24-36)."""
    _fields_ = [("max_tokens", ctypes.c_int), ("temperature", ctypes.c_float), ("top_p", ctypes.c_float),
                ("top_k", ctypes.c_int), ("repetition_penalty", ctypes.c_float), ("has_seed", ctypes.c_int),
                ("seed", ctypes.c_ulonglong), ("system_prompt", ctypes.c_char_p),
                ("stop_strings", ctypes.c_void_p), ("stop_count", ctypes.c_int), ("tier_id", ctypes.c_int)]


def _eng_err(what):
    raise RuntimeError(f"{what}: {lib().g4dense_engine_last_error().decode()}")


class Engine:
    """The engine behind include/g4dense/c_api.h (greedy or sampled, optional drafter)."""

    def __init__(self, target=None, preset=None, seed=0, centered=False, draft=None, draft_preset=None,
                 draft_seed=1, draft_k=0, max_context=4096, kv_bf16=False, tp_rank=0, tp_size=1,
                 nccl_id=None, device=-1, gate_min_accept=0.45, gate_window=24, tokenizer_path=None):
        L = lib()
        cfg = EngineConfig()
        L.g4dense_config_default(ctypes.byref(cfg))
        self._keep = []
        def cstr(x):
            if x is None:
                return None
            b = str(x).encode()
            self._keep.append(b)
            return b
        cfg.container_path = cstr(target)
        cfg.synthetic_preset = cstr(preset)
        cfg.synthetic_seed = seed
        cfg.synthetic_centered = 1 if centered else 0
        cfg.draft_path = cstr(draft)
        cfg.draft_preset = cstr(draft_preset)
        cfg.draft_seed = draft_seed
        cfg.draft_k = draft_k
        cfg.max_context = max_context
        cfg.kv_bf16 = 1 if kv_bf16 else 0
        cfg.tp_rank, cfg.tp_size = tp_rank, tp_size
        if nccl_id is not None:
            self._nid = ctypes.create_string_buffer(bytes(nccl_id), 128)
            cfg.nccl_unique_id = ctypes.cast(self._nid, ctypes.c_void_p)
        cfg.device = device
        cfg.gate_min_accept = gate_min_accept
        cfg.gate_window = gate_window
        cfg.tokenizer_path = cstr(tokenizer_path)
        self.h = L.g4dense_engine_create_ex(ctypes.byref(cfg))
        if not self.h:
            _eng_err("g4dense_engine_create_ex")

    def set_decode_options(self, stop_token=-1, draft_k=-1, replay=None, mismatch_rate=0.0, mismatch_seed=0):
        r = None if replay is None else np.ascontiguousarray(replay, np.uint32)
        if lib().g4dense_engine_set_decode_options(self.h, stop_token, draft_k,
                                                   None if r is None else r.ctypes.data_as(_vp),
                                                   0 if r is None else len(r), mismatch_rate, mismatch_seed):
            _eng_err("g4dense_engine_set_decode_options")

    def set_device_sampling(self, on):
        if lib().g4dense_engine_set_device_sampling(self.h, 1 if on else 0):
            _eng_err("g4dense_engine_set_device_sampling")

    def generate(self, prompt, max_tokens, temperature=0.0, top_p=1.0, top_k=0, seed=None, callback=None,
                 repetition_penalty=1.0):
        o = GenOptions()
        lib().g4dense_options_default(ctypes.byref(o))
        o.max_tokens = max_tokens
        o.temperature, o.top_p, o.top_k = temperature, top_p, top_k
        o.repetition_penalty = repetition_penalty
        o.has_seed = 0 if seed is None else 1
        o.seed = 0 if seed is None else seed
        p = np.ascontiguousarray(prompt, np.uint32)
        cb = TOKEN_CB(lambda u, i, t, d: int(callback(t)) if callback else 1)
        r = lib().g4dense_engine_generate_tokens(self.h, p.ctypes.data_as(_vp), len(p), ctypes.byref(o), cb, None)
        if r is None:
            _eng_err("g4dense_engine_generate_tokens")
        out = np.zeros(max_tokens + 32, np.uint32)
        n = lib().g4dense_engine_last_tokens(self.h, out.ctypes.data_as(_vp), len(out))
        return out[:n].copy()

    def generate_text(self, prompt, use_chat_template=True, max_tokens=512, temperature=0.0, top_p=1.0, top_k=0,
                      seed=None, callback=None, options=None):
        """ForwardRunner::generate(prompt, options) through g4dense_engine_generate_text: returns the
        concatenated pieces (bytes); callback(token, piece_bytes) -> bool continues. `options`
        (a GenOptions) overrides the keyword sampling arguments."""
        o = options
        if o is None:
            o = GenOptions()
            lib().g4dense_options_default(ctypes.byref(o))
            o.max_tokens = max_tokens
            o.temperature, o.top_p, o.top_k = temperature, top_p, top_k
            o.has_seed = 0 if seed is None else 1
            o.seed = 0 if seed is None else seed
        cb = TOKEN_CB(lambda u, i, t, d: int(callback(t, d)) if callback else 1)
        r = lib().g4dense_engine_generate_text(self.h, _as_bytes(prompt), 1 if use_chat_template else 0,
                                               ctypes.byref(o), cb, None)
        if r is None:
            _eng_err("g4dense_engine_generate_text")
        return r

    def tokens(self, cap=1 << 16):
        out = np.zeros(cap, np.uint32)
        n = lib().g4dense_engine_last_tokens(self.h, out.ctypes.data_as(_vp), cap)
        return out[:n].copy()

    def tokenizer(self):
        """The engine's own tokenizer (None when it loaded none)."""
        t = lib().g4dense_engine_tokenizer(self.h)
        return Tokenizer(_handle=t, _owner=self) if t else None

    def rounds(self, cap=4096):
        buf = np.zeros(3 * cap, np.int32)
        n = lib().g4dense_engine_last_rounds(self.h, buf.ctypes.data_as(_vp), cap)
        return [tuple(int(v) for v in buf[3 * i:3 * i + 3]) for i in range(n)]

    def forward_batch(self, tokens, base, vocab=None, all_positions=True):
        t = np.ascontiguousarray(tokens, np.uint32)
        out = None
        if vocab is not None:
            out = np.zeros((len(t) if all_positions else 1, vocab), np.float32)
        rc = lib().g4dense_engine_forward_batch(self.h, t.ctypes.data_as(_vp), len(t), base,
                                                None if out is None else out.ctypes.data_as(_vp),
                                                1 if all_positions else 0)
        if rc:
            _eng_err("g4dense_engine_forward_batch")
        return out

    def mtp_draft(self, seed_token, context_length, hidden_row, k, vocab):
        """Greedy MTP drafting from the target's current state: (tokens [k], logits [k][vocab])."""
        toks = np.zeros(k, np.uint32)
        logits = np.zeros((k, vocab), np.float32)
        if lib().g4dense_engine_mtp_draft(self.h, seed_token, context_length, hidden_row, k,
                                          toks.ctypes.data_as(_vp), logits.ctypes.data_as(_vp)):
            _eng_err("g4dense_engine_mtp_draft")
        return toks, logits

    def draft_steps(self, token, pos, k, vocab=None):
        """Greedy drafting by the separate drafter: k chained one-row steps from `token` at position
        `pos` -> (tokens [k], logits [k][vocab] or None)."""
        toks = np.zeros(k, np.uint32)
        logits = None if vocab is None else np.zeros((k, vocab), np.float32)
        if lib().g4dense_engine_draft_steps(self.h, token, pos, k, toks.ctypes.data_as(_vp),
                                            None if logits is None else logits.ctypes.data_as(_vp)):
            _eng_err("g4dense_engine_draft_steps")
        return toks, logits

    STAT_KEYS = ("emitted", "decode_gpu_ms", "ttft_ms", "total_ms", "drafted", "accepted", "rounds",
                 "gated_steps", "launches", "h2d_bytes", "d2h_bytes", "decode_wall_ms")

    def stats(self):
        buf = np.zeros(len(self.STAT_KEYS), np.float64)
        n = lib().g4dense_engine_last_stats(self.h, buf.ctypes.data_as(_vp), len(buf))
        return dict(zip(self.STAT_KEYS[:n], buf[:n].tolist()))

    def set_gate(self, min_accept=0.45, window=24):
        if lib().g4dense_engine_set_gate(self.h, min_accept, window):
            _eng_err("g4dense_engine_set_gate")

    def time_pass(self, which, batch, reps=5, pos=0):
        ms = lib().g4dense_engine_time_pass(self.h, which, batch, pos, reps)
        if ms < 0:
            _eng_err("g4dense_engine_time_pass")
        return ms

    def profile_gemms(self, batch, reps=3):
        b = ctypes.c_ulonglong(0)
        n = ctypes.c_int(0)
        ms = lib().g4dense_engine_profile_gemms(self.h, batch, reps, ctypes.byref(b), ctypes.byref(n))
        if ms < 0:
            _eng_err("g4dense_engine_profile_gemms")
        return ms, int(b.value), int(n.value)

    def telemetry(self):
        import json
        return json.loads(lib().g4dense_engine_get_telemetry(self.h).decode())

    def close(self):
        if getattr(self, "h", None):
            lib().g4dense_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _as_bytes(x):
    return x if isinstance(x, bytes) else str(x).encode()


def _take(ptr, n):
    if not ptr:
        raise RuntimeError(lib().g4dense_engine_last_error().decode())
    return ctypes.string_at(ptr, n.value)


class Tokenizer:
    """The engine's tokenizer (g4dense_tokenizer_*): Gemma-4 tokenizer.json BPE, chat template,
    byte-fallback decoding. Text goes in as str or UTF-8 bytes and comes out as bytes."""

    def __init__(self, path=None, arch=0, _handle=None, _owner=None):
        self._owner = _owner
        if _handle is not None:
            self.h = _handle
            return
        self.h = lib().g4dense_tokenizer_open(None if path is None else str(path).encode(), arch)
        if not self.h:
            _eng_err("g4dense_tokenizer_open")

    def encode(self, text, add_bos=True):
        b = _as_bytes(text)
        n = lib().g4dense_tokenizer_encode(self.h, b, len(b), 1 if add_bos else 0, None, 0)
        if n < 0:
            _eng_err("g4dense_tokenizer_encode")
        out = np.zeros(max(n, 1), np.uint32)
        n = lib().g4dense_tokenizer_encode(self.h, b, len(b), 1 if add_bos else 0, out.ctypes.data_as(_vp), len(out))
        return out[:n].tolist()

    def decode(self, ids, skip_special=True):
        a = np.ascontiguousarray(ids, np.uint32)
        n = ctypes.c_size_t(0)
        return _take(lib().g4dense_tokenizer_decode(self.h, a.ctypes.data_as(_vp), len(a), 1 if skip_special else 0,
                                                    ctypes.byref(n)), n)

    def decode_single(self, tid, skip_special=True):
        n = ctypes.c_size_t(0)
        return _take(lib().g4dense_tokenizer_decode_single(self.h, tid, 1 if skip_special else 0, ctypes.byref(n)), n)

    def chat_template(self, messages):
        """messages: a JSON string, or [(role, content)] / [{"role": .., "content": ..}]."""
        import json
        if not isinstance(messages, (str, bytes)):
            messages = json.dumps([m if isinstance(m, dict) else {"role": m[0], "content": m[1]} for m in messages])
        r = lib().g4dense_tokenizer_chat_template(self.h, _as_bytes(messages))
        if r is None:
            _eng_err("g4dense_tokenizer_chat_template")
        return r

    def special_ids(self):
        v = np.zeros(6, np.uint32)
        lib().g4dense_tokenizer_special_ids(self.h, v.ctypes.data_as(_vp))
        return dict(zip(("bos", "eos", "pad", "unk", "end_of_turn", "vocab_size"), v.tolist()))

    def stop_ids(self):
        v = np.zeros(16, np.uint32)
        n = lib().g4dense_tokenizer_stop_ids(self.h, v.ctypes.data_as(_vp), len(v))
        return v[:n].tolist()

    def byte_value(self, tid):
        b = ctypes.c_ubyte(0)
        return b.value if lib().g4dense_tokenizer_byte_value(self.h, tid, ctypes.byref(b)) else None

    def is_special(self, tid):
        return bool(lib().g4dense_tokenizer_is_special(self.h, tid))

    def detokenizer(self, skip_special=True):
        return Detokenizer(self, skip_special)

    def close(self):
        if getattr(self, "h", None) and self._owner is None:
            lib().g4dense_tokenizer_destroy(self.h)
        self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Detokenizer:
    """IncrementalDetokenizer: push(id) -> bytes now complete; finish() -> the rest."""

    def __init__(self, tok: Tokenizer, skip_special=True):
        self._tok = tok
        self.h = lib().g4dense_detokenizer_create(tok.h, 1 if skip_special else 0)
        if not self.h:
            _eng_err("g4dense_detokenizer_create")

    def push(self, tid):
        n = ctypes.c_size_t(0)
        return _take(lib().g4dense_detokenizer_push(self.h, tid, ctypes.byref(n)), n)

    def finish(self):
        n = ctypes.c_size_t(0)
        return _take(lib().g4dense_detokenizer_finish(self.h, ctypes.byref(n)), n)

    def __del__(self):
        try:
            if self.h:
                lib().g4dense_detokenizer_destroy(self.h)
        except Exception:
            pass


class StopMatcher:
    """StreamingStopMatcher over byte strings."""

    def __init__(self, stops):
        arr = (ctypes.c_char_p * max(1, len(stops)))(*[_as_bytes(s) for s in stops])
        self.h = lib().g4dense_stop_matcher_create(arr, len(stops))
        if not self.h:
            _eng_err("g4dense_stop_matcher_create")

    def push(self, text):
        b = _as_bytes(text)
        n = ctypes.c_size_t(0)
        return _take(lib().g4dense_stop_matcher_push(self.h, b, len(b), ctypes.byref(n)), n)

    def finish(self):
        n = ctypes.c_size_t(0)
        return _take(lib().g4dense_stop_matcher_finish(self.h, ctypes.byref(n)), n)

    @property
    def stopped(self):
        return bool(lib().g4dense_stop_matcher_stopped(self.h, None))

    @property
    def matched(self):
        m = ctypes.c_char_p()
        lib().g4dense_stop_matcher_stopped(self.h, ctypes.byref(m))
        return m.value or b""

    def __del__(self):
        try:
            if self.h:
                lib().g4dense_stop_matcher_destroy(self.h)
        except Exception:
            pass


def utf8_repair(data: bytes, flush_all: bool):
    """-> (repaired bytes, bytes of `data` consumed)."""
    used, n = ctypes.c_size_t(0), ctypes.c_size_t(0)
    p = lib().g4dense_utf8_repair(data, len(data), 1 if flush_all else 0, ctypes.byref(used), ctypes.byref(n))
    return ctypes.string_at(p, n.value), used.value


def validate_container(path) -> str:
    """Checks a container's header against its file with the engine loader's rules (no GPU
    needed). Returns "g4dense" or "g4mtp"; raises ValueError listing every broken rule."""
    rc = lib().g4dense_container_validate(str(path).encode())
    if rc < 0:
        raise ValueError(lib().g4dense_engine_last_error().decode())
    return {1: "g4dense", 2: "g4mtp"}[rc]
