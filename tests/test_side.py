"""The int8 / elementwise side kernels: GemvInt8 (shaders/GemvInt8.hlsl:13-33) and AttnGate
(shaders/AttnGate.hlsl:15-32), against the CPU oracle (oracle/g4d_oracle.c)."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O


def bf16_bits(x):
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def test_oracle_attn_gate_formula():
    rng = np.random.default_rng(0)
    ctx, gate = rng.normal(0, 2, 257).astype(np.float32), rng.normal(0, 4, 257).astype(np.float32)
    want = ctx.astype(np.float64) / (1.0 + np.exp(-gate.astype(np.float64)))
    assert np.allclose(O.attn_gate(ctx, gate), want, rtol=1e-6, atol=1e-7)


def test_oracle_int8_gemv_matches_float64():
    rng = np.random.default_rng(1)
    rows, K = 7, 192
    q = rng.integers(0, 256, (rows, K), dtype=np.uint8)
    s, b = bf16_bits(np.abs(rng.normal(0, 0.02, (rows, K // 64)))), bf16_bits(rng.normal(0, 0.01, (rows, K // 64)))
    x = rng.normal(0, 1, K).astype(np.float32)
    sf = (s.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    bf = (b.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    w = q.astype(np.float64) * np.repeat(sf, 64, axis=1) + np.repeat(bf, 64, axis=1)
    want = w @ x.astype(np.float64)
    got = O.int8_gemv(q.view(np.uint32), s, b, x)
    assert np.allclose(got, want, rtol=1e-5, atol=1e-5 * np.abs(w).sum(axis=1).max())


@pytest.mark.gpu
@pytest.mark.parametrize("rows,K", [(1, 64), (8, 1536), (37, 5376), (1000, 2112)])
def test_gemv_int8_matches_oracle(built_lib, rows, K):
    import torch
    from g4dense_b200.api import gemv_int8
    rng = np.random.default_rng(rows + K)
    q = rng.integers(0, 256, (rows, K), dtype=np.uint8)
    s, b = bf16_bits(np.abs(rng.normal(0, 0.02, (rows, K // 64)))), bf16_bits(rng.normal(0, 0.01, (rows, K // 64)))
    x = rng.normal(0, 1, K).astype(np.float32)
    want = O.int8_gemv(q.view(np.uint32), s, b, x)
    out = torch.empty(rows, device="cuda")
    gemv_int8(torch.from_numpy(q).cuda(), torch.from_numpy(s.view(np.int16)).cuda(),
              torch.from_numpy(b.view(np.int16)).cuda(), torch.from_numpy(x).cuda(), out)
    got = out.cpu().numpy()
    sf = (s.astype(np.uint32) << 16).view(np.float32)
    scale = (q.astype(np.float64) * np.repeat(sf, 64, axis=1) + np.abs(np.repeat((b.astype(np.uint32) << 16)
             .view(np.float32), 64, axis=1))) @ np.abs(x).astype(np.float64)
    # Summation order differs from the oracle's sequential row walk: 1e-5 of sum |w * x|.
    assert np.all(np.abs(got - want) <= 1e-5 * scale + 1e-6)


@pytest.mark.gpu
def test_attn_gate_matches_oracle(built_lib):
    import torch
    from g4dense_b200.api import attn_gate
    rng = np.random.default_rng(2)
    batch, n, ld = 5, 8192, 8200
    ctx = rng.normal(0, 1, (batch, ld)).astype(np.float32)
    gate = rng.normal(0, 3, (batch, ld)).astype(np.float32)
    tc, tg = torch.from_numpy(ctx).cuda(), torch.from_numpy(gate).cuda()
    out = torch.zeros(batch, ld, device="cuda")
    attn_gate(tc[:, :n], tg[:, :n], out[:, :n])
    got = out.cpu().numpy()
    want = np.stack([O.attn_gate(ctx[m, :n], gate[m, :n]) for m in range(batch)])
    # expf differs from the host's exp by at most a couple of ulp.
    assert np.allclose(got[:, :n], want, rtol=4e-7, atol=1e-30)
    assert np.all(got[:, n:] == 0)
