"""Profiling drivers: run one piece of the hot path inside a CUDA profiler range so an external
profiler started with `--profile-from-start off` sees exactly that piece.

    python -m g4dense_b200.profile pass  --which target|draft|mtp --batch M --pos P [--layers L]
                                         [--ctx C] [--kv-bf16]
        one forward pass of the 31B-shaped target (or the E2B-shaped drafter) with M rows at
        positions P..P+M-1 (attention spans P earlier cache entries), after 5 timed warm
        passes; prints their mean CUDA-event time. `mtp`: one step of the 31B assistant's MTP
        drafter (M = 1) attending the target's P cached positions. `draftstep`: chained one-row
        E2B-shaped drafter steps from position P, as a speculative round runs them.
    python -m g4dense_b200.profile gemms [--only NAME] [--batch M]
        each distinct verify-GEMM shape of the 31B pass once (the kernel as the pass runs it:
        split-K slots left for the consuming epilogue), through the g4b_qmat C-ABI.
    python -m g4dense_b200.profile pgemm [--only NAME] [--batch M] [--reps R]
        each distinct GEMM shape of a 31B prefill chunk of M (17..128) rows on the tcgen05
        prefill GEMM: CUDA-event time per launch (mean of R after 3 warm launches), the
        algorithmic rate 2*M*N*K / time, and the weighted sum over one prefill pass; then
        one launch per shape inside the profiler range.

Synthetic weights; nothing here is on the product path."""
from __future__ import annotations

import argparse
import ctypes
import json
import sys

import numpy as np

# (name, N, K) of every distinct verify GEMM in a Gemma-4-31B pass (50 sliding + 10 global
# layers + the tied LM head).
GEMM_SHAPES = [("qkv_sliding", 16384, 5376), ("qkv_global", 18432, 5376), ("o_sliding", 5376, 8192),
               ("o_global", 5376, 16384), ("gateup", 43008, 5376), ("down", 5376, 21504),
               ("lm_head", 262144, 5376)]
# Launches of each shape per pass.
GEMM_COUNTS = {"qkv_sliding": 50, "qkv_global": 10, "o_sliding": 50, "o_global": 10, "gateup": 60, "down": 60,
               "lm_head": 1}


def _profiler():
    cu = ctypes.CDLL("libcuda.so.1")
    return cu.cuProfilerStart, cu.cuProfilerStop


def run_pass(which, batch, pos, layers=0, ctx=4096, kv_bf16=False):
    from .api import Engine
    slot = 0
    if which == "target":
        preset = "gemma4-31b" + (f":layers={layers}" if layers else "")
        e = Engine(preset=preset, seed=0, max_context=ctx, kv_bf16=kv_bf16, device=0)
    elif which == "mtp":
        e = Engine(preset="gemma4-31b", seed=0, draft_preset="gemma4-31b-assistant", draft_seed=2, max_context=4096,
                   device=0)
        slot = 2
    elif which == "draftstep":
        # Chained one-row E2B-shaped drafter steps, as a speculative round runs them. The small
        # target only hosts the drafter.
        e = Engine(preset="config0-target", seed=0, draft_preset="gemma4-e2b", draft_seed=1, max_context=4096,
                   device=0)
        slot = 3
        batch = 1
    else:
        e = Engine(preset="gemma4-e2b", seed=1, max_context=4096, device=0)
    ms = e.time_pass(slot, batch, 20 if which == "draftstep" else 5, pos=pos)
    start, stop = _profiler()
    start()
    e.time_pass(slot, batch, 1, pos=pos)
    stop()
    e.close()
    print(json.dumps({"which": which, "batch": batch, "pos": pos, "ms_per_pass": ms}))


def run_gemms(only, batch):
    import torch
    from .api import QMat
    rng = np.random.default_rng(0)
    mats = []
    for name, N, K in GEMM_SHAPES:
        if only and name != only:
            continue
        W = torch.from_numpy(rng.integers(0, 2**32, (N, K // 8), dtype=np.uint32).view(np.int32)).cuda()
        S = torch.full((N, K // 64), 0x3C00, dtype=torch.int16, device="cuda")
        B = torch.zeros((N, K // 64), dtype=torch.int16, device="cuda")
        q = QMat(W, S, B)
        del W, S, B
        x = torch.randn(batch, K, device="cuda")
        y = torch.empty(batch, N, device="cuda")
        q.gemm(x, y)
        mats.append((name, q))
    torch.cuda.synchronize()
    start, stop = _profiler()
    start()
    for _, q in mats:
        q.run_partial(batch)
    torch.cuda.synchronize()
    stop()
    for _, q in mats:
        q.check_error()
    print(json.dumps({"gemms": [n for n, _ in mats], "batch": batch}))


def _make_qmat(rng, N, K):
    import torch
    from .api import QMat
    W = torch.from_numpy(rng.integers(0, 2**32, (N, K // 8), dtype=np.uint32).view(np.int32)).cuda()
    S = torch.full((N, K // 64), 0x3C00, dtype=torch.int16, device="cuda")
    B = torch.zeros((N, K // 64), dtype=torch.int16, device="cuda")
    return QMat(W, S, B)


def run_pgemm(only, batch, reps):
    import torch
    rng = np.random.default_rng(0)
    rows, mats = [], []
    pass_us = 0.0
    for name, N, K in GEMM_SHAPES:
        if (only and name != only) or (not only and name == "lm_head"):
            continue  # a prefill chunk ranks only its last row: the LM head runs on one row
        q = _make_qmat(rng, N, K)
        x = torch.randn(batch, K, device="cuda")
        y = torch.empty(batch, N, device="cuda")
        q.prepare(x)
        for _ in range(3):
            q.run(batch, y)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        for _ in range(reps):
            q.run(batch, y)
        ev1.record()
        torch.cuda.synchronize()
        q.check_error()
        us = ev0.elapsed_time(ev1) * 1000.0 / reps
        tflops = 2.0 * batch * N * K / (us * 1e-6) / 1e12
        pass_us += us * GEMM_COUNTS[name]
        rows.append({"gemm": name, "N": N, "K": K, "us": round(us, 2), "tflops": round(tflops, 1)})
        mats.append((q, y))
    start, stop = _profiler()
    start()
    for q, y in mats:
        q.run(batch, y)
    torch.cuda.synchronize()
    stop()
    print(json.dumps({"batch": batch, "shapes": rows, "prefill_pass_gemm_ms": round(pass_us / 1000.0, 3)}))


def main(argv=None):
    ap = argparse.ArgumentParser(prog="python -m g4dense_b200.profile")
    sub = ap.add_subparsers(dest="cmd", required=True)
    p = sub.add_parser("pass")
    p.add_argument("--which", choices=["target", "draft", "mtp", "draftstep"], default="target")
    p.add_argument("--ctx", type=int, default=4096, help="KV capacity (target)")
    p.add_argument("--kv-bf16", action="store_true", help="bf16 KV cache (target, long-context mode)")
    p.add_argument("--batch", type=int, default=5)
    p.add_argument("--pos", type=int, default=768)
    p.add_argument("--layers", type=int, default=0, help="target layers (0 = all 60); a small case for ncu")
    g = sub.add_parser("gemms")
    g.add_argument("--only", default=None)
    g.add_argument("--batch", type=int, default=5)
    pg = sub.add_parser("pgemm")
    pg.add_argument("--only", default=None)
    pg.add_argument("--batch", type=int, default=128)
    pg.add_argument("--reps", type=int, default=20)
    a = ap.parse_args(argv)
    if a.cmd == "pass":
        run_pass(a.which, a.batch, a.pos, a.layers, a.ctx, a.kv_bf16)
    elif a.cmd == "pgemm":
        run_pgemm(a.only, a.batch, a.reps)
    else:
        run_gemms(a.only, a.batch)
    return 0


if __name__ == "__main__":
    sys.exit(main())
