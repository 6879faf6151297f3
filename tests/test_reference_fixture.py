"""The reference's own test fixture, tests/fixtures/tiny.g4dense (CPU only).

container.reference_tiny_container() restates the reference's fixture generator
(tools/make_synthetic_model.py): Gaussian weights quantized per group by their range, unit norms,
GQA 2, a 1024-entry vocabulary. tests/golden/tiny.json (made by tests/golden/make_tiny_golden.py)
holds the sha256 of the file that generator writes and the reference CPU runner's logits on it,
over a 40-token prompt and its 24-token greedy continuation (input-dependent tokens, unlike the
BASELINE config-0 model). The restatement must write the same bytes. The engine's loader and the
verifier must accept the file. The oracle must reproduce the reference runner's logits bit for
bit at every position.
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np

from g4dense_b200 import api
from g4dense_b200 import container as C
from g4dense_b200 import verify as W
from oracle import oracle as O

GOLDEN = json.loads((Path(__file__).parent / "golden" / "tiny.json").read_text())


def _fixture(tmp_path) -> Path:
    path = tmp_path / "tiny.g4dense"
    path.write_bytes(C.reference_tiny_container())
    return path


def test_restatement_writes_the_reference_fixture(tmp_path):
    path = _fixture(tmp_path)
    assert hashlib.sha256(path.read_bytes()).hexdigest() == GOLDEN["container_sha256"]
    assert api.validate_container(path) == "g4dense"
    info = W.verify_container(path)
    assert (info["layers"], info["d_model"], info["kv_heads"], info["vocab_size"]) == (4, 256, 2, 1024)


def test_oracle_matches_reference_runner_on_the_fixture(tmp_path):
    m = O.RestatedModel(str(_fixture(tmp_path)))
    try:
        for p, (tok, want) in enumerate(zip(GOLDEN["tokens"], GOLDEN["positions"])):
            logits = np.asarray(m.forward(tok, p), dtype=np.float32)
            assert hashlib.sha256(logits.tobytes()).hexdigest() == want["sha256"], f"position {p}"
            assert int(np.argmax(logits)) == want["argmax"]
    finally:
        m.close()
    prompt_len = len(GOLDEN["prompt"])
    assert GOLDEN["tokens"][:prompt_len] == GOLDEN["prompt"]
    # The continuation is the argmax chain, and it is not one repeated token.
    cont = GOLDEN["tokens"][prompt_len:]
    assert cont == [GOLDEN["positions"][p]["argmax"] for p in range(prompt_len - 1, len(GOLDEN["tokens"]) - 1)]
    assert len(set(cont)) > len(cont) // 2
