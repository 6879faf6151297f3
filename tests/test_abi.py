"""The drop-in boundary, checked without a GPU: the library loads, exports every symbol the
headers declare, and the no-device parts of the C API behave like the reference's
(src/c_api.cpp: nullptr / -1 with last_error set, "{}" telemetry for a null handle,
options_default values)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]


def declared_symbols():
    syms = set()
    for h in (REPO / "include").rglob("*.h"):
        text = h.read_text()
        for m in re.finditer(r"(?:G4DENSE_API|G4B_API)\s+[\w\s\*]+?\b(\w+)\s*\(", text):
            syms.add(m.group(1))
    return syms


def test_headers_declare_reference_api():
    syms = declared_symbols()
    # include/g4dense/c_api.h:18-49 of the reference
    for s in ["g4dense_engine_create", "g4dense_engine_destroy", "g4dense_engine_generate",
              "g4dense_engine_get_telemetry", "g4dense_options_default", "g4dense_engine_generate_ex",
              "g4dense_engine_last_stop_reason", "g4dense_engine_last_error", "g4dense_engine_switch_tier",
              "g4dense_engine_stop"]:
        assert s in syms, s


def test_library_exports_every_declared_symbol(built_lib):
    lib = ctypes.CDLL(str(built_lib))
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_options_struct_layout_and_defaults(built_lib):
    from g4dense_b200.api import GenOptions, lib
    L = lib()
    # G4DenseGenerationOptions must stay binary-identical to the reference's struct
    # (include/g4dense/c_api.h:24-36): 56 bytes on LP64, seed at offset 24.
    assert ctypes.sizeof(GenOptions) == 56
    assert GenOptions.seed.offset == 24 and GenOptions.tier_id.offset == 52
    o = GenOptions()
    L.g4dense_options_default(ctypes.byref(o))
    assert (o.max_tokens, round(o.temperature, 4), round(o.top_p, 4), o.top_k) == (512, 0.2, 0.95, 64)
    assert (o.repetition_penalty, o.has_seed, o.seed, o.stop_count, o.tier_id) == (1.0, 0, 0, 0, 1)


def test_null_handle_behaviour(built_lib):
    from g4dense_b200.api import lib
    L = lib()
    assert L.g4dense_engine_get_telemetry(None) == b"{}"
    assert L.g4dense_engine_generate(None, b"hi", 8) is None
    assert b"Invalid handle" in L.g4dense_engine_last_error()
    assert L.g4dense_engine_switch_tier(None, 1) == -1
    assert L.g4dense_engine_last_stop_reason(None) == 0
    L.g4dense_engine_stop(None)
    L.g4dense_engine_destroy(None)


def test_create_missing_container_fails_loudly(built_lib, tmp_path):
    from g4dense_b200.api import lib
    L = lib()
    h = L.g4dense_engine_create(str(tmp_path / "missing.g4dense").encode())
    assert h is None
    assert L.g4dense_engine_last_error() != b""


def test_c_header_compiles_with_reference_layout(tmp_path):
    """The header is plain C and the struct layout matches what the reference's callers use."""
    import subprocess
    src = tmp_path / "probe.c"
    src.write_text(
        "#include <stddef.h>\n#include \"g4dense/c_api.h\"\n#include \"g4dense_b200_ops.h\"\n"
        "_Static_assert(sizeof(G4DenseGenerationOptions) == 56, \"size\");\n"
        "_Static_assert(offsetof(G4DenseGenerationOptions, seed) == 24, \"seed\");\n"
        "_Static_assert(offsetof(G4DenseGenerationOptions, tier_id) == 52, \"tier\");\n"
        "int main(void) { return 0; }\n")
    r = subprocess.run(["gcc", "-std=c11", "-I", str(REPO / "include"), "-o", str(tmp_path / "probe"), str(src)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_engine_config_layout_matches_header(tmp_path):
    """The Python mirror of G4DenseEngineConfig has the C struct's size and field offsets."""
    import subprocess
    from g4dense_b200.api import EngineConfig
    fields = [f[0] for f in EngineConfig._fields_]
    src = tmp_path / "cfg.c"
    src.write_text("#include <stdio.h>\n#include <stddef.h>\n#include \"g4dense/c_api.h\"\nint main(void) {\n"
                   + "".join(f'  printf("%zu\\n", offsetof(G4DenseEngineConfig, {f}));\n' for f in fields)
                   + '  printf("%zu\\n", sizeof(G4DenseEngineConfig));\n  return 0;\n}\n')
    exe = tmp_path / "cfg"
    r = subprocess.run(["gcc", "-std=c11", "-I", str(REPO / "include"), "-o", str(exe), str(src)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    got = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    want = [getattr(EngineConfig, f).offset for f in fields] + [ctypes.sizeof(EngineConfig)]
    assert got == want
