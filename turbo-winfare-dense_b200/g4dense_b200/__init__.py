"""Python host mirror of the B200 speculative-decode library.

The product is the native library ``lib/libg4dense_b200.so`` (CUDA kernels for sm_100a plus
the C++ runner behind the reference's C API). This package only binds it with ctypes for
tests and benchmarks, and writes synthetic containers. Importing it never compiles anything;
``g4dense_b200.build.build()`` does.
"""
from .api import lib, LIB_PATH, QMat, Engine, GenOptions  # noqa: F401
