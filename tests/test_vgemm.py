"""Verify GEMM (GemmInt4Batch / GemvInt4 semantics) against the CPU oracle.

The oracle is oracle/g4d_oracle.c's g4o_int4_gemm: full-precision dequantization q*s+b and a
sequential fp32 dot per row (src/cpu_reference.cpp:94-138). The GPU sums in a different order
with fp16 hi/lo activation operands, so the bar is a bound relative to the row's absolute
mass: |gpu - ref| <= 2e-6 * sum_k |w_k x_k| + 1e-30, far inside the reference's own kernel
tolerances (GemvInt4 1e-3/1e-3, GemmInt4Batch 1e-3/1e-2, tests/test_gpu_kernels.cpp:345,584).
"""
from __future__ import annotations

import numpy as np
import pytest

REL_TOL = 2e-6


def make_matrix(rng, N, K, centered=False):
    from g4dense_b200.container import random_quant_block
    return random_quant_block(rng, N, K, centered)


def dequant(W, S, B):
    from g4dense_b200.container import bf16_bits_to_f32
    N, K = W.shape[0], W.shape[1] * 8
    nib = np.stack([(W >> (4 * j)) & 0xF for j in range(8)], axis=-1).reshape(N, K).astype(np.float64)
    s = np.repeat(bf16_bits_to_f32(S).astype(np.float64), 64, axis=1)
    b = np.repeat(bf16_bits_to_f32(B).astype(np.float64), 64, axis=1)
    return nib * s + b


def check_gemm(N, K, M, seed=0, centered=False, x_scale=1.0):
    import torch
    from g4dense_b200 import QMat
    from oracle import oracle as O

    rng = np.random.default_rng(seed)
    W, S, B = make_matrix(rng, N, K, centered)
    x = (rng.standard_normal((M, K), dtype=np.float32) * x_scale).astype(np.float32)
    dev = torch.device("cuda:0")
    Wt = torch.from_numpy(W.view(np.int32)).to(dev)
    St = torch.from_numpy(S.view(np.int16)).to(dev)
    Bt = torch.from_numpy(B.view(np.int16)).to(dev)
    q = QMat(Wt, St, Bt)
    xt = torch.from_numpy(x).to(dev)
    out = torch.full((M, N), float("nan"), device=dev)
    q.gemm(xt, out)
    torch.cuda.synchronize()
    q.check_error()
    got = out.cpu().numpy()
    ref = O.int4_gemm(W, S, B, x)
    mass = np.abs(x.astype(np.float64)) @ np.abs(dequant(W, S, B)).T
    err = np.abs(got.astype(np.float64) - ref) / (mass + 1e-30)
    assert np.isfinite(got).all()
    assert err.max() <= REL_TOL, f"N={N} K={K} M={M}: max rel err {err.max():.3e}"
    # Run twice: the split-K counters must have been reset by the first launch.
    out2 = torch.full((M, N), float("nan"), device=dev)
    q.gemm(xt, out2)
    torch.cuda.synchronize()
    assert np.array_equal(out2.cpu().numpy(), got), "second launch differs (determinism)"
    q.close()
    return err.max()


@pytest.mark.gpu
@pytest.mark.parametrize("M", [1, 2, 4, 5, 8, 9, 10, 11, 16])
def test_vgemm_small_shapes(built_lib, M):
    # N not a multiple of 256 (partial CTA row group), K with a padded half k-tile.
    check_gemm(320, 192, M, seed=M)
    check_gemm(64, 256, M, seed=100 + M, centered=True)


@pytest.mark.gpu
@pytest.mark.parametrize("K,N", [(5376, 1024), (21504, 256), (1536, 6144)])
@pytest.mark.parametrize("M", [1, 5, 9, 16])
def test_vgemm_model_shapes(built_lib, K, N, M):
    check_gemm(N, K, M, seed=K + N + M)


@pytest.mark.gpu
def test_vgemm_activation_range(built_lib):
    # Large and tiny activations exercise the per-group power-of-two scaling.
    check_gemm(256, 512, 5, seed=7, x_scale=3.0e4)
    check_gemm(256, 512, 5, seed=8, x_scale=1.0e-5)


@pytest.mark.gpu
def test_vgemm_rejects_bad_args(built_lib):
    import torch
    from g4dense_b200 import QMat
    dev = torch.device("cuda:0")
    W = torch.zeros((64, 12), dtype=torch.int32, device=dev)  # K = 96, not a multiple of 64
    S = torch.zeros((64, 1), dtype=torch.int16, device=dev)
    with pytest.raises(RuntimeError):
        QMat(W, S, S)



def bf16_round(x):
    from g4dense_b200.container import bf16_bits_to_f32, f32_to_bf16_bits
    return bf16_bits_to_f32(f32_to_bf16_bits(x)).reshape(x.shape)


@pytest.mark.gpu
@pytest.mark.parametrize("K,N", [(5376, 21504), (21504, 5376), (5376, 8192), (5376, 262144)])
def test_vgemm_config1_shapes(built_lib, K, N):
    """BASELINE config 1 at its own shapes: bf16 activations ~N(0, 1) of M in {1, 2, 5, 8, 16}
    rows times INT4 G64 weights [N, K] with the container's distributions, fp32 output, with
    the real split-K slot counts. The oracle's sequential fp32 dot (src/cpu_reference.cpp:94-138)
    runs on a subset of rows -- the first and last 64-row groups, a row straddling every
    256-row boundary sampled, and 256 random rows -- sliced out of the same matrix, so the
    check is exact per row; every row must be finite and a second launch bit-identical."""
    import torch
    from g4dense_b200 import QMat
    from oracle import oracle as O

    rng = np.random.default_rng(K * 7 + N)
    W, S, B = make_matrix(rng, N, K)
    rows = np.unique(np.concatenate([np.arange(64), np.arange(N - 64, N), rng.integers(0, N, 256),
                                     np.arange(255, N, max(256, N // 64))]))
    Wr, Sr, Br = W[rows], S[rows], B[rows]
    mass_w = np.abs(dequant(Wr, Sr, Br))
    dev = torch.device("cuda:0")
    q = QMat(torch.from_numpy(W.view(np.int32)).to(dev), torch.from_numpy(S.view(np.int16)).to(dev),
             torch.from_numpy(B.view(np.int16)).to(dev))
    del W
    worst = 0.0
    for M in (1, 2, 5, 8, 16):
        x = bf16_round(rng.standard_normal((M, K), dtype=np.float32))
        xt = torch.from_numpy(x).to(dev)
        out = torch.full((M, N), float("nan"), device=dev)
        q.gemm(xt, out)
        out2 = torch.full((M, N), float("nan"), device=dev)
        q.gemm(xt, out2)
        torch.cuda.synchronize()
        q.check_error()
        assert bool(torch.isfinite(out).all()), f"M={M}: non-finite outputs"
        assert torch.equal(out, out2), f"M={M}: second launch differs"
        got = out[:, torch.from_numpy(rows).to(dev)].cpu().numpy()
        ref = O.int4_gemm(Wr, Sr, Br, x)
        mass = np.abs(x.astype(np.float64)) @ mass_w.T
        err = (np.abs(got.astype(np.float64) - ref) / (mass + 1e-30)).max()
        assert err <= REL_TOL, f"K={K} N={N} M={M}: max rel err {err:.3e}"
        worst = max(worst, err)
    print(f"config-1 K={K} N={N}: {len(rows)} rows x M in 1,2,5,8,16 checked, worst rel err {worst:.2e}")
    q.close()
