"""g4b_qmat_run_noalloc: the verify GEMM with the library's static split-K scratch.

It runs the same kernel, grid and slot order as g4b_qmat_run, so two calls in a row must both
reproduce g4b_qmat_run bit for bit. A matrix whose launch needs more scratch than the static
buffer holds is rejected with a clear error. This file is named to run last, and it also passes
on its own."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def make_qmat(N, K, seed):
    import torch
    from g4dense_b200.api import QMat
    rng = np.random.default_rng(seed)
    W = torch.from_numpy(rng.integers(0, 2**32, (N, K // 8), dtype=np.uint32).view(np.int32)).cuda()
    # bf16 scales ~|N(0, 0.02)| and biases ~N(0, 0.01), as in the container recipe
    s = np.abs(rng.normal(0, 0.02, (N, K // 64))).astype(np.float32).view(np.uint32) >> 16
    b = rng.normal(0, 0.01, (N, K // 64)).astype(np.float32).view(np.uint32) >> 16
    S = torch.from_numpy(s.astype(np.uint16).view(np.int16)).cuda()
    B = torch.from_numpy(b.astype(np.uint16).view(np.int16)).cuda()
    return QMat(W, S, B)


@pytest.mark.parametrize("N,K,M", [(5376, 8192, 5), (8192, 5376, 1), (4096, 21504, 16), (1000, 320, 3)])
def test_noalloc_matches_run_on_two_calls(built_lib, N, K, M):
    import torch
    q = make_qmat(N, K, seed=N + K + M)
    x = torch.randn(M, K, device="cuda")
    q.prepare(x)
    ref = torch.empty(M, N, device="cuda")
    q.run(M, ref)
    outs = [torch.full((M, N), float("nan"), device="cuda") for _ in range(2)]
    torch.cuda.synchronize()
    free0, alloc0 = torch.cuda.mem_get_info()[0], torch.cuda.memory_allocated()
    for call in range(2):
        q.run_noalloc(M, outs[call])
        torch.cuda.synchronize()
    # The property the entry point exists for: the calls reserve no device memory.
    assert torch.cuda.mem_get_info()[0] == free0 and torch.cuda.memory_allocated() == alloc0
    for call, got in enumerate(outs):
        assert torch.equal(got, ref), f"call {call}: max |diff| {(got - ref).abs().max().item()}"
    q.check_error()
    q.close()


def test_noalloc_rejects_prefill_rows(built_lib):
    import torch
    q = make_qmat(256, 128, seed=3)
    x = torch.randn(17, 128, device="cuda")
    q.prepare(x)
    out = torch.empty(17, 256, device="cuda")
    with pytest.raises(RuntimeError, match="M must be 1..16"):
        q.run_noalloc(17, out)
    q.close()


def test_noalloc_rejects_oversized_scratch(built_lib):
    import torch
    # 512 row groups x 2 slots x 16 KiB = 16 MiB of split-K scratch at M = 5: over the 8 MiB buffer.
    q = make_qmat(131072, 64, seed=1)
    x = torch.randn(5, 64, device="cuda")
    q.prepare(x)
    out = torch.empty(5, 131072, device="cuda")
    with pytest.raises(RuntimeError, match="static buffer holds 8 MiB"):
        q.run_noalloc(5, out)
    q.run(5, out)  # the allocating entry point still serves it
    torch.cuda.synchronize()
    q.close()
