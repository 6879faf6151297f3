"""Tensor parallelism: 2 ranks, one GPU each, run the config-0 target with query heads, FFN
columns and the vocabulary split (KV heads replicated where there are fewer than ranks); the
o-projection and down-projection partials are summed across ranks over peer memory and the LM
head's per-chunk bests all-gathered over NCCL. Greedy token streams and round records must equal
the oracle's (the reference has no multi-GPU path; its single-process CPU runner is the oracle).
A 200-token prompt also runs the tensor-core prefill (chunks of 128 and 72 rows) under TP."""
from __future__ import annotations

import json
import os
import subprocess
import sys

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def gpu_count():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


@pytest.mark.parametrize("spec,plen", [("no_spec", 24), ("spec_k5", 24), ("spec_k5", 200)])
def test_tp2_streams_match_oracle(built_lib, config0, tmp_path, spec, plen):
    if gpu_count() < 2:
        pytest.skip("needs 2 GPUs")
    tgt, drf = config0["target"], config0["draft"]
    n = 48
    prompt = np.random.default_rng(0).integers(0, 4096, plen)
    D = O.RestatedModel(drf) if spec == "spec_k5" else None
    want_tokens, want_rounds = O.spec_generate(O.RestatedModel(tgt), D, prompt, n, verify_width=5)
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29533",
           os.path.join(REPO, "tests", "tp_worker.py"), str(tgt), str(drf) if D else "-", "5", str(plen), str(n),
           str(tmp_path)]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stderr[-3000:]
    for rank in range(2):
        got = json.loads((tmp_path / f"rank{rank}.json").read_text())
        assert got["tokens"] == want_tokens.tolist(), f"rank {rank} tokens"
        assert [tuple(x) for x in got["rounds"]] == [tuple(x) for x in want_rounds], f"rank {rank} rounds"
