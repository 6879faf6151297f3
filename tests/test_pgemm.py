"""Prefill GEMM (17..128 rows on the tcgen05 tensor cores) against the CPU oracle.

Same oracle and bar as the verify GEMM (test_vgemm.py): oracle/g4d_oracle.c's g4o_int4_gemm
(full-precision q*s+b, sequential fp32 dot, src/cpu_reference.cpp:94-138), and
|gpu - ref| <= 2e-6 * sum_k |w_k x_k|. The shapes cover the three ways a 128-row weight tile is
finished: by one CTA alone (written straight to the output), split across a few CTAs, and split
across dozens (the last CTA to arrive adds every slot in slot order). Each case runs twice and
must repeat bit for bit, which also checks that the per-tile counters were reset.
"""
from __future__ import annotations

import pytest

from test_vgemm import check_gemm


@pytest.mark.gpu
@pytest.mark.parametrize("M", [17, 31, 48, 100, 128])
def test_pgemm_small_shapes(built_lib, M):
    # N not a multiple of 128 (partial last tile); K = 192 is three groups (a padded k-tile).
    check_gemm(320, 192, M, seed=M)
    check_gemm(128, 256, M, seed=100 + M, centered=True)


@pytest.mark.gpu
@pytest.mark.parametrize("M", [24, 128])
def test_pgemm_tile_ownership(built_lib, M):
    # Many tiles, few groups: most tiles are wholly one CTA's.
    check_gemm(32768, 192, M, seed=7 + M)
    # Two tiles over a long K: each tile's groups spread over ~74 CTAs.
    check_gemm(256, 21504, M, seed=8 + M)


@pytest.mark.gpu
@pytest.mark.parametrize("K,N", [(5376, 1024), (1536, 6144), (8192, 5376)])
@pytest.mark.parametrize("M", [64, 128])
def test_pgemm_model_shapes(built_lib, K, N, M):
    check_gemm(N, K, M, seed=K + N + M)


@pytest.mark.gpu
def test_pgemm_large_activations(built_lib):
    # Activations spanning many binades: the per-(group, row) power-of-two scale keeps the
    # hi/lo split exact to ~2^-22 of each group's largest element.
    check_gemm(512, 1024, 96, seed=3, x_scale=1e4)
    check_gemm(512, 1024, 96, seed=4, x_scale=1e-4)
