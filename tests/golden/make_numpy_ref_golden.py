"""Writes tests/golden/numpy_ref.json: the logits of the REFERENCE's independent NumPy forward pass
(tools/numpy_reference.py, run unmodified from the reference checkout as its own process) for every
synthetic checkpoint of g4dense_b200.synth_checkpoint.forward_cases().

Run from the repository root where the reference checkout exists:
    python tests/golden/make_numpy_ref_golden.py [REFERENCE_ROOT]

That tool reads the MLX checkpoint directly (config.json + safetensors) and runs every layer in
float32, one position at a time; `--save-dir` makes it write each position's softcapped logits.
Per case the fixture stores the prompt, the digest of the input tensors and each position's
logits as little-endian float16 in base64 (|logit| <= 30, so the rounding is at most 0.008).
"""
from __future__ import annotations

import base64
import json
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[2]
sys.path[:0] = [str(REPO), str(REPO / "turbo-winfare-dense_b200")]

from g4dense_b200 import synth_checkpoint as S  # noqa: E402

OUT = Path(__file__).resolve().parent / "numpy_ref.json"


def main(ref_root: str) -> None:
    tool = Path(ref_root) / "tools" / "numpy_reference.py"
    golden = {}
    with tempfile.TemporaryDirectory() as tmp:
        for name, (config, tensors, prompt) in S.forward_cases().items():
            ck = S.write_checkpoint(Path(tmp) / name, config, tensors, prefix="model.")
            save = Path(tmp) / f"{name}_logits"
            layers = config["text_config"]["num_hidden_layers"]
            subprocess.run([sys.executable, str(tool), "--ckpt", str(ck), "--layers", str(layers),
                            "--tokens", ",".join(map(str, prompt)), "--save-dir", str(save),
                            "--dump-dir", str(Path(tmp) / "no_dumps")], check=True, capture_output=True)
            rows = [np.fromfile(save / f"token{p}_logits.bin", dtype=np.float32) for p in range(len(prompt))]
            golden[name] = {"tensors": S.tensors_digest(tensors), "prompt": prompt,
                            "logits_f16": [base64.b64encode(r.astype("<f2").tobytes()).decode() for r in rows]}
            print(name, [int(np.argmax(r)) for r in rows])
    OUT.write_text(json.dumps(golden, indent=1) + "\n")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else str(REPO.parent / "reference"))
