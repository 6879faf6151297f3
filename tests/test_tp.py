"""Tensor parallelism: 2, 4 or 8 ranks, one GPU each, run container.TP_TEST_TARGET (8 query
heads; 8 KV heads on the sliding layers, split by rank; 2 KV heads on the full-attention layer,
replicated at TP = 8 as the 31B's four-head global layers are) with query heads, FFN columns and
the vocabulary split. The o-projection and down-projection partials are summed across ranks over
peer memory and the LM head's per-chunk bests all-gathered over NCCL.

Zero-mean weights and pinned prompts (container.TP_PINNED*), whose oracle margins along the whole
stream stay clear of the FP16 K/V rounding noise, so greedy token streams and round records must
equal the oracle's exactly (the reference has no multi-GPU path; its single-process CPU runner,
restated in oracle/ and pinned to the reference by tests/test_oracle.py, is the oracle). Cases:
no drafter; the target drafting for itself (every draft accepted); the config-3 replay drafter at
a 0.25 mismatch rate (accepts and rejects mixed); a 300-token prompt that also runs the
tensor-core prefill (chunks of 128, 128 and 44 rows) under TP; and temperature-0.8 speculative
decoding with rejection sampling, whose verify logits are all-gathered from the ranks' vocabulary
slices before the reference's acceptance test runs (BASELINE-distribution weights, which the GPU
reproduces to ~1e-5, with a near drafter so that drafts are both accepted and rejected). The
long-context attention (tensor cores, bf16 KV, head_dim 512 full-attention layer) also runs under
TP, on the 31B attention geometry, its logits compared with the oracle's."""
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


@pytest.fixture(scope="module")
def tp_model(tmp_path_factory):
    from g4dense_b200 import container as C
    return C.write_container(tmp_path_factory.mktemp("tp") / "tp_target.g4dense", C.TP_TEST_TARGET,
                             seed=C.TP_TEST_SEED, centered=True)


@pytest.fixture(scope="module")
def tp_sampled_pair(tmp_path_factory):
    from g4dense_b200 import container as C
    d = tmp_path_factory.mktemp("tp_sampled")
    tgt = C.write_container(d / "tp_base.g4dense", C.TP_TEST_TARGET, seed=C.TP_TEST_SEED)
    near = C.perturbed_copy(tgt, d / "tp_near.g4dense", C.TP_TEST_TARGET, 0.0, seed=C.NEAR_DRAFT_SEED,
                            embed_frac=C.NEAR_DRAFT_EMBED_FRAC)
    return tgt, near


def _run_ranks(world, tmp_path, args, env_extra=None):
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={29533 + world}",
           os.path.join(REPO, "tests", "tp_worker.py")] + args
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", **(env_extra or {}))
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stderr[-3000:]
    return [json.loads((tmp_path / f"rank{rank}.json").read_text()) for rank in range(world)]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_sampled_spec_matches_oracle(built_lib, tp_sampled_pair, tmp_path, world):
    if gpu_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from g4dense_b200 import container as C
    tgt, near = tp_sampled_pair
    t, tp, tk, seed = C.SAMPLED_PARAMS
    prompt = C.tp_pinned_prompt()
    want_tokens, want_rounds = O.spec_generate(O.RestatedModel(tgt), O.RestatedModel(near), prompt, 48, verify_width=5,
                                               sampling=O.Sampling(t, tp, tk, 1.0, 1, seed))
    np.save(tmp_path / "prompt.npy", np.asarray(prompt, np.uint32))
    got = _run_ranks(world, tmp_path, [str(tgt), str(near), "5", str(tmp_path / "prompt.npy"), "48", str(tmp_path)],
                     {"G4B_TEST_SAMPLING": f"{t},{tp},{tk},{seed}"})
    for rank, g in enumerate(got):
        assert g["tokens"] == want_tokens.tolist(), f"rank {rank} tokens"
        assert [tuple(x) for x in g["rounds"]] == [tuple(x) for x in want_rounds], f"rank {rank} rounds"
    print(f"TP={world} sampled: compared {len(want_tokens)} tokens and {len(want_rounds)} rounds "
          f"({sum(r[1] for r in want_rounds)}/{sum(r[0] for r in want_rounds)} drafts accepted) on each rank")


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("case", ["no_spec", "self_k5", "replay_k5", "long_self_k5"])
def test_tp_streams_match_oracle(built_lib, config0, tp_model, tmp_path, world, case):
    if gpu_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from g4dense_b200 import container as C
    long = case.startswith("long")
    prompt = C.tp_pinned_prompt(long)
    n = C.TP_PINNED_LONG[2] if long else C.TP_PINNED[2]
    T = O.RestatedModel(tp_model)
    extra, gate = [], 24
    if case == "no_spec":
        dpath = None
    elif case == "replay_k5":
        dpath = config0["draft_centered"]
        stream, _ = O.spec_generate(T, None, prompt, n)
        np.save(tmp_path / "replay.npy", np.asarray(stream, np.uint32))
        extra, gate = [str(tmp_path / "replay.npy"), "0.25", "9"], -1
    else:
        dpath = tp_model
    D = O.RestatedModel(dpath) if dpath else None
    want_tokens, want_rounds = O.spec_generate(
        T, D, prompt, n, verify_width=5, gate_window=gate,
        replay_stream=stream if extra else None, mismatch_rate=0.25 if extra else 0.0, mismatch_seed=9)
    if case == "replay_k5":
        assert any(0 < r[1] < r[0] for r in want_rounds)
    np.save(tmp_path / "prompt.npy", np.asarray(prompt, np.uint32))
    ranks = _run_ranks(world, tmp_path, [str(tp_model), str(dpath) if dpath else "-", "5",
                                         str(tmp_path / "prompt.npy"), str(n), str(tmp_path)] + extra)
    for rank, got in enumerate(ranks):
        assert got["tokens"] == want_tokens.tolist(), f"rank {rank} tokens"
        assert [tuple(x) for x in got["rounds"]] == [tuple(x) for x in want_rounds], f"rank {rank} rounds"
    print(f"TP={world} {case} prompt {len(prompt)}: compared {len(want_tokens)} tokens and {len(want_rounds)} "
          f"rounds on each of {world} ranks")


@pytest.mark.parametrize("world", [2, 4])
def test_tp_long_context_attention_matches_oracle(built_lib, geom31, tmp_path, world):
    """The 31B attention geometry at toy width (head_dim 512 full-attention layer, one KV head,
    replicated across ranks) with a bf16 KV cache and the tensor-core long-context attention on
    every rank: prefill chunks and verify batches, logits gathered from the ranks' vocabulary
    slices, within 2e-2 of the row's max of the oracle's."""
    if gpu_count() < world:
        pytest.skip(f"needs {world} GPUs")
    path = geom31["baseline"]
    chunks = [128, 128, 100, 9, 16, 128, 51, 1]
    toks = np.random.default_rng(34).integers(0, 4096, sum(chunks))
    np.save(tmp_path / "prompt.npy", np.asarray(toks, np.uint32))
    _run_ranks(world, tmp_path, [str(path), "-", "5", str(tmp_path / "prompt.npy"), "0", str(tmp_path)],
               {"G4DENSE_ATTN_LC": "1", "G4B_TEST_LC_LOGITS": ",".join(map(str, chunks)), "G4B_TEST_VOCAB": "4096"})
    ref = O.RestatedModel(path, max_ctx=1024, kv_mode=O.KV_BF16)
    want = [ref.forward(int(t), p) for p, t in enumerate(toks)]
    data = np.load(tmp_path / "logits.npz")
    pos, worst = 0, 0.0
    for i, m in enumerate(chunks):
        got = data[f"arr_{i}"]
        rows = range(m) if m <= 16 else [m - 1]
        for j, r in enumerate(rows):
            g, w = got[j], want[pos + r]
            d = np.abs(g.astype(np.float64) - w).max() / np.abs(w).max()
            assert np.isfinite(g).all() and d <= 2e-2, f"TP={world} pass {i} row {r}: {d:.3e}"
            worst = max(worst, d)
            srt = np.sort(w)
            if srt[-1] - srt[-2] >= 2e-2 * np.abs(w).max():
                assert int(np.argmax(g)) == int(np.argmax(w)), f"TP={world} pass {i} row {r}: argmax"
        pos += m
    print(f"TP={world} long-context attention: worst |diff| / max |logit| = {worst:.2e}")
