"""Writes tests/golden/convert.json: the REFERENCE converters' output, run unmodified from the
reference checkout -- tools/convert_hf_to_g4dense.py for every synthetic checkpoint of
g4dense_b200.synth_checkpoint.converter_cases() (section "model") and tools/convert_hf_assistant.py
for every one of assistant_cases() (section "assistant").

Run from the repository root where the reference checkout exists:
    python tests/golden/make_convert_golden.py [REFERENCE_ROOT]

Per case it stores the digest of the input tensors (so a test can tell a changed synthetic
checkpoint from a converter bug) and either the SHA-256 and size of the container written, or
`"refused": true` when the reference converter raised.
"""
from __future__ import annotations

import contextlib
import hashlib
import importlib.util
import io
import json
import sys
import tempfile
from pathlib import Path

REPO = Path(__file__).resolve().parents[2]
sys.path[:0] = [str(REPO), str(REPO / "turbo-winfare-dense_b200")]

from g4dense_b200 import synth_checkpoint as S  # noqa: E402

OUT = Path(__file__).resolve().parent / "convert.json"


def _load(path: Path, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _run(cases: dict, convert, tmp: Path) -> dict:
    golden = {}
    for name, (config, tensors, prefix, shards, _) in cases.items():
        ck = S.write_checkpoint(tmp / name, config, tensors, prefix, shards)
        out = tmp / f"{name}.out"
        entry = {"tensors": S.tensors_digest(tensors)}
        try:
            with contextlib.redirect_stdout(io.StringIO()):
                convert(str(ck), str(out))
            data = out.read_bytes()
            entry.update(sha256=hashlib.sha256(data).hexdigest(), size=len(data))
        except Exception as e:  # the reference raises ValueError / KeyError / FileNotFoundError
            entry.update(refused=True, error=type(e).__name__)
        golden[name] = entry
        print(name, entry.get("sha256", entry.get("error")))
    return golden


def main(ref_root: str) -> None:
    tools = Path(ref_root) / "tools"
    model = _load(tools / "convert_hf_to_g4dense.py", "ref_convert")
    assistant = _load(tools / "convert_hf_assistant.py", "ref_convert_assistant")
    with tempfile.TemporaryDirectory() as tmp:
        golden = {"model": _run(S.converter_cases(), model.convert_checkpoint, Path(tmp)),
                  "assistant": _run(S.assistant_cases(), assistant.convert_assistant_checkpoint, Path(tmp))}
    OUT.write_text(json.dumps(golden, indent=1) + "\n")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else str(REPO.parent / "reference"))
