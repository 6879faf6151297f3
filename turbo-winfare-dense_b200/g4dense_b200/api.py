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
        L.g4b_qmat_check_error.argtypes = [_vp]
        _bind_engine(L)
        _lib = L
    return _lib


def _bind_engine(L):
    """Binds the engine-level C API when the library exports it."""
    if not hasattr(L, "g4dense_engine_create"):
        return
    L.g4dense_engine_last_error.restype = ctypes.c_char_p
    L.g4dense_engine_create.restype = _vp
    L.g4dense_engine_create.argtypes = [ctypes.c_char_p]
    L.g4dense_engine_destroy.argtypes = [_vp]
    L.g4dense_engine_get_telemetry.restype = ctypes.c_char_p
    L.g4dense_engine_get_telemetry.argtypes = [_vp]
    L.g4dense_options_default.argtypes = [_vp]


def _check(rc, what):
    if rc != 0:
        raise RuntimeError(f"{what} failed ({rc}): {lib().g4b_last_error().decode()}")


def _dptr(t):
    """Device pointer of a torch CUDA tensor."""
    return ctypes.c_void_p(t.data_ptr())


def _stream(stream):
    return ctypes.c_void_p(stream.cuda_stream if stream is not None else 0)


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


class Engine:
    """Placeholder until the engine C API is bound (see _bind_engine)."""
