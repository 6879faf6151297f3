"""Device-side token sampling (csrc/sample.cu) against the oracle's sample_token.

The oracle (oracle/g4d_oracle.c g4o_sample_token) restates the reference's sample_token
(src/sampling.cpp:92-169) and is itself pinned to the reference's compiled code
(tests/test_oracle.py). The device draw must pick the same token for the same logits row,
parameters and seed: the shortlist, the top-p cut and the draw follow the reference's order;
only the fp64 denominator is summed in a different order, which can matter only for a draw
within a few ulps of a boundary (none in these cases). Then the engine's non-speculative
sampled loop is run with the device draw and with the host draw over copied logits: the
streams must be identical.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O

from test_engine import engine

CASES = [
    # (temperature, top_p, top_k)
    (0.0, 1.0, 0),     # greedy
    (0.8, 1.0, 0),     # temperature only: the reference's 256-wide shortlist
    (0.7, 0.9, 40),
    (1.2, 0.95, 256),
    (0.5, 1.0, 8),
    (2.0, 0.5, 1),
]


def _logits(rng, V, kind):
    if kind == "normal":
        return (rng.standard_normal(V) * 3).astype(np.float32)
    if kind == "flat":
        return (rng.standard_normal(V) * 0.05).astype(np.float32)
    if kind == "ties":  # many equal values: ties must resolve to the lower index
        return (np.round(rng.standard_normal(V) * 4) / 2).astype(np.float32)
    if kind == "peaked":
        x = (rng.standard_normal(V) * 0.5).astype(np.float32)
        x[rng.integers(0, V, 3)] = 25.0
        return x
    raise ValueError(kind)


@pytest.mark.gpu
@pytest.mark.parametrize("V", [7, 1000, 4096, 5000, 262144])
@pytest.mark.parametrize("kind", ["normal", "flat", "ties", "peaked"])
def test_device_draw_matches_oracle(built_lib, V, kind):
    import torch
    from g4dense_b200 import api

    lib = O.restated_lib()
    rng = np.random.default_rng(V * 7 + len(kind))
    ws = torch.zeros(api.sample_workspace_bytes(), dtype=torch.uint8, device="cuda")
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    for trial in range(12):
        logits = _logits(rng, V, kind)
        t, p, k = CASES[trial % len(CASES)]
        seed = int(rng.integers(1, 2 ** 63))
        d = torch.from_numpy(logits).cuda()
        api.sample_token(d, t, p, k, seed, ws, out)
        got = int(out.item()) & 0xFFFFFFFF
        want = lib.g4o_sample_token(logits.ctypes.data, V, O.Sampling(t, p, k, 1.0, 1, 9), seed)
        assert got == want, (V, kind, trial, (t, p, k))


@pytest.mark.gpu
def test_device_draw_rejects_bad_arguments(built_lib):
    import torch
    from g4dense_b200 import api

    ws = torch.zeros(api.sample_workspace_bytes(), dtype=torch.uint8, device="cuda")
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    x = torch.zeros(16, device="cuda")
    with pytest.raises(RuntimeError, match="bad arguments"):
        api.sample_token(x, 0.8, 1.0, 257, 1, ws, out)
    with pytest.raises(RuntimeError, match="bad arguments"):
        api.sample_token(x, 0.8, 0.0, 4, 1, ws, out)


@pytest.mark.gpu
@pytest.mark.parametrize("params", [(0.8, 1.0, 0, 1.0), (0.7, 0.9, 40, 1.0), (1.5, 1.0, 4, 1.0),
                                    (0.9, 1.0, 0, 1.3), (1.2, 0.95, 64, 0.8)])
def test_sampled_loop_device_equals_host(built_lib, config0, params):
    """The device draw (with the repetition penalty applied on the device when it is not 1)
    against the host draw over the copied logits row: the same stream."""
    t, p, k, pen = params
    prompt = np.random.default_rng(11).integers(0, 4096, 20)
    prompt[5:9] = prompt[0]  # repeated ids: the penalty compounds
    e = engine(config0["target_centered"])
    dev = e.generate(prompt, 40, temperature=t, top_p=p, top_k=k, seed=17, repetition_penalty=pen)
    e.set_device_sampling(False)
    host = e.generate(prompt, 40, temperature=t, top_p=p, top_k=k, seed=17, repetition_penalty=pen)
    assert dev.tolist() == host.tolist()
    e.close()
