"""Writes tests/golden/tiny.json: the reference's own test fixture and its CPU runner's answers on it.

* `container_sha256`: of tests/fixtures/tiny.g4dense as the REFERENCE's generator writes it
  (tools/make_synthetic_model.py, run unmodified with its defaults: seed 42, Gemma-4);
* per position of a 40-token seeded prompt followed by the greedy continuation (24 tokens): the
  REFERENCE's CpuReferenceRunner logits (oracle/_ref, built from src/cpu_reference.cpp) as the
  sha256 of their fp32 bytes, the argmax, the top-5 and the top-1 minus top-2 margin.

Run from the repository root where the reference checkout exists (oracle/_ref must be built):
    python tests/golden/make_tiny_golden.py [REFERENCE_ROOT]
"""
from __future__ import annotations

import hashlib
import json
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[2]
sys.path[:0] = [str(REPO), str(REPO / "turbo-winfare-dense_b200")]

from oracle import oracle as O  # noqa: E402

OUT = Path(__file__).resolve().parent / "tiny.json"
PROMPT_LEN, GREEDY = 40, 24


def main(ref_root: str) -> None:
    with tempfile.TemporaryDirectory() as tmp:
        path = Path(tmp) / "tiny.g4dense"
        subprocess.run([sys.executable, str(Path(ref_root) / "tools" / "make_synthetic_model.py"), "--out", str(path)],
                       check=True, capture_output=True)
        prompt = [int(t) for t in np.random.default_rng(11).integers(0, 1024, PROMPT_LEN)]
        ref = O.ReferenceModel(str(path))
        tokens, positions = list(prompt), []
        for p in range(PROMPT_LEN + GREEDY):
            logits = np.asarray(ref.forward(tokens[p], p), dtype=np.float32)
            order = np.argsort(-logits, kind="stable")
            positions.append({"sha256": hashlib.sha256(logits.tobytes()).hexdigest(), "argmax": int(order[0]),
                              "top5": [int(i) for i in order[:5]],
                              "margin": float(logits[order[0]] - logits[order[1]])})
            if p + 1 >= len(tokens):
                tokens.append(int(order[0]))
        ref.close()
        golden = {"container_sha256": hashlib.sha256(path.read_bytes()).hexdigest(), "prompt": prompt,
                  "tokens": tokens[:PROMPT_LEN + GREEDY], "positions": positions}
    OUT.write_text(json.dumps(golden, indent=1) + "\n")
    print("greedy continuation:", tokens[PROMPT_LEN:])


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else str(REPO.parent / "reference"))
