"""Long-context attention on the tensor cores (csrc/attn_lc.cu): the full-attention layers'
verify-batch attention in long-context mode (bf16 KV, head_dim 512).

* Against the oracle (`oracle/g4d_oracle.c` in bf16-KV mode, pinned to the reference's runner):
  the 31B attention geometry at toy width (a head_dim 512 full-attention layer with GQA 4) over
  700 positions fed as verify batches of 1..16 rows, every row's logits within 2e-2 of the row's
  max (top-1 and top-5 exact where the margins allow). The split count is forced down (1 and 3)
  so each CTA runs several 128-key tiles (the double-buffered scores, the output accumulated
  across tiles, the rescale when a row's maximum rises), and left at its natural value.
* Prefill chunks of 17..128 rows (blocks of up to 48 positions of one query head) against the
  oracle: each chunk's last-row logits and the verify rows that read the keys the chunks wrote.
* Against the cluster kernel (`csrc/attention.cu`) at the 31B's real shapes: a 6-layer cut whose
  8 192-token bf16 context is prefilled in 128-row chunks, then verify batches of 9, 1 and 16
  rows; the two kernels' logits agree to 2e-3 of the row's max.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

REL_TOL = 2e-2


def check_logits(got, ref, where, tol=REL_TOL):
    d = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    scale = np.abs(ref).max()
    assert np.isfinite(got).all(), where
    assert d.max() <= tol * scale, f"{where}: max |diff| {d.max():.3e} vs max |logit| {scale:.3f}"
    tie = tol * scale
    srt = np.sort(ref)[::-1]
    if srt[0] - srt[1] >= tie:
        assert int(np.argmax(got)) == int(np.argmax(ref)), where
        top = np.argsort(-ref, kind="stable")[:6]
        if np.all(np.diff(ref[top]) <= -tie):
            assert list(np.argsort(-got, kind="stable")[:5]) == list(top[:5]), where
    return d.max() / scale


@pytest.mark.parametrize("splits", [1, 3, 0])
def test_lc_attention_matches_oracle(built_lib, geom31, monkeypatch, splits):
    from g4dense_b200 import Engine
    monkeypatch.setenv("G4DENSE_ATTN_LC", "1")
    if splits:
        monkeypatch.setenv("G4DENSE_ATTN_LC_SPLITS", str(splits))
    path = geom31["baseline"]
    e = Engine(target=path, max_context=1024, kv_bf16=True)
    ref = O.RestatedModel(path, max_ctx=1024, kv_mode=O.KV_BF16)
    toks = np.random.default_rng(31).integers(0, 4096, 700)
    want = [ref.forward(int(t), p) for p, t in enumerate(toks)]
    plan = [16, 9, 1, 5, 12, 16, 16, 2] * 12
    pos, worst = 0, 0.0
    for m in plan:
        m = min(m, len(toks) - pos)
        if m == 0:
            break
        got = e.forward_batch(toks[pos:pos + m], pos, vocab=4096, all_positions=True)
        for i in range(m):
            worst = max(worst, check_logits(got[i], want[pos + i], f"splits {splits}: position {pos + i} (batch {m})"))
        pos += m
    assert pos == len(toks)
    e.close()
    print(f"splits {splits or 'natural'}: {pos} positions, worst |diff| / max |logit| = {worst:.2e}")


def test_lc_matches_cluster_kernel_31b_long_context(built_lib, monkeypatch):
    from g4dense_b200 import Engine
    ctx, V = 8192, 262144
    toks = np.random.default_rng(32).integers(0, V, ctx + 16)
    outs = {}
    for lc in ("0", "1"):
        monkeypatch.setenv("G4DENSE_ATTN_LC", lc)
        e = Engine(preset="gemma4-31b:layers=6", seed=3, centered=True, max_context=16384, kv_bf16=True)
        for pos in range(0, ctx, 128):
            e.forward_batch(toks[pos:pos + 128], pos, vocab=None, all_positions=False)
        # each batch rewrites the ring slots of positions ctx.. with the same keys
        outs[lc] = [e.forward_batch(toks[ctx:ctx + m], ctx, vocab=V, all_positions=True) for m in (9, 1, 16)]
        e.close()
    worst = 0.0
    for m, a, b in zip((9, 1, 16), outs["0"], outs["1"]):
        for i in range(m):
            worst = max(worst, check_logits(b[i], a[i], f"batch {m} row {i}", tol=2e-3))
    print(f"tensor-core vs cluster attention at {ctx} keys: worst |diff| / max |logit| = {worst:.2e}")


@pytest.mark.parametrize("splits", [1, 0])
def test_lc_prefill_chunks_match_oracle(built_lib, geom31, monkeypatch, splits):
    """Prefill chunks of 17..128 rows: the rows run as blocks of up to 48 positions of one query
    head, each with its own causal key limit; the chunk's last-row logits and the verify rows that
    follow (reading the keys the chunks wrote) against the oracle."""
    from g4dense_b200 import Engine
    monkeypatch.setenv("G4DENSE_ATTN_LC", "1")
    if splits:
        monkeypatch.setenv("G4DENSE_ATTN_LC_SPLITS", str(splits))
    path = geom31["baseline"]
    e = Engine(target=path, max_context=1024, kv_bf16=True)
    ref = O.RestatedModel(path, max_ctx=1024, kv_mode=O.KV_BF16)
    toks = np.random.default_rng(33).integers(0, 4096, 700)
    want = [ref.forward(int(t), p) for p, t in enumerate(toks)]
    pos, worst = 0, 0.0
    for m in [128, 17, 100, 64, 9, 128, 49, 5, 96, 16, 88]:
        m = min(m, len(toks) - pos)
        if m > 16:
            got = e.forward_batch(toks[pos:pos + m], pos, vocab=4096, all_positions=False)
            worst = max(worst, check_logits(got[0], want[pos + m - 1], f"prefill chunk at {pos} (rows {m})"))
        else:
            got = e.forward_batch(toks[pos:pos + m], pos, vocab=4096, all_positions=True)
            for i in range(m):
                worst = max(worst, check_logits(got[i], want[pos + i], f"position {pos + i} (batch {m})"))
        pos += m
    assert pos == len(toks)
    e.close()
    print(f"prefill chunks, splits {splits or 'natural'}: worst |diff| / max |logit| = {worst:.2e}")
