#!/usr/bin/env python
"""Benchmark: BASELINE's "31B spec-decode tok/s at 1/2/4/8 B200; verify-GEMM HBM GB/s vs peak".

Workload: Gemma-4-31B-shaped INT4 G64 target (60 layers, d 5376, 32/16
heads, head_dim 256, global layers 512/4 every 6th from 5, FFN 21504, vocab 262144) and an
E2B-shaped drafter (35 layers, d 1536, 8/1 heads, head_dim 256, FFN 6144), synthetic weights
with the container's value distributions generated on the device (seed 0 / 1). Greedy
speculative decoding with k = 4 drafts (verify width 5), KV sized for 4096, a 512-token
uniform-random prompt (seed 0) and 256 generated tokens per request.

Acceptance is set by config 3's oracle drafter: the drafter model runs its k steps (cost) and
its proposals replay the target's own greedy stream with i.i.d. injected mismatches. The
headline uses a 0.25 mismatch rate; the line also carries the {0, 0.25, 0.5, 1.0} sweep and
the natural random-weight drafter (which the adaptive gate switches off after 24 drafts). The
adaptive gate is off for the replay runs, whose acceptance the replay sets.

One step = one generation request. `value` = decoded tokens / device decode time (CUDA events
on the engine's stream from the end of prefill to the last token, max over ranks); `e2e` =
tokens / wall time of the C-API call with host prompt and host output (prefill, host<->device
copies and the per-round result reads included). `roofline` = the verify GEMM (the dominant
kernel): algorithmic bytes of one 5-row verify pass's GEMMs / their CUDA-event time, against
the measured HBM copy bandwidth in MEASURED_PEAKS.json.

The line also carries BASELINE config 1 (`config1`: the verify GEMM alone at its (K, N) x M grid,
GB/s per cell) and config 4 (`long_context`: 32768-token bf16 KV after a 30000-token prefill,
verify width 9, greedy and temperature-0.8 rejection sampling, at the run's TP size), and the
speculative weight-bytes bound of the measured rounds.

`--impl reference` times the reference's own CPU code (oracle/_ref, src/cpu_reference.cpp built
unmodified) on a bounded sample of the same workload on the host: a 31B-shaped container with
one sliding and one global layer plus the full embedding / LM head, one position per step,
extrapolated to 60 layers by weight bytes. It is single-threaded, as the reference is.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "turbo-winfare-dense_b200"))

METRIC = "31B spec-decode tok/s"
UNIT = "tok/s"
PROMPT_LEN, GEN_LEN, VERIFY_WIDTH, MISMATCH = 512, 256, 5, 0.25
# Weight bytes of one 31B verify pass (50 sliding + 10 global layers + LM head, INT4 G64).
B31_PASS_BYTES = 50 * 269.40e6 + 10 * 300.37e6 + 792.72e6
# Weight bytes of one E2B-shaped drafter step (35 layers + LM head).
E2B_STEP_BYTES = 35 * 19.91e6 + 226.5e6
# (K, N) of the verify-GEMM sweep and its verify widths.
CONFIG1_SHAPES = [(5376, 21504), (21504, 5376), (5376, 8192), (5376, 262144)]
CONFIG1_M = [1, 2, 5, 8, 16]


def peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def clocks_start(path):
    cmd = ["nvidia-smi", "--query-gpu=index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
           "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
           "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
           "--format=csv,noheader,nounits", "-lms", "200"]
    try:
        return subprocess.Popen(cmd, stdout=open(path, "w"), stderr=subprocess.DEVNULL)
    except Exception:
        return None


def clocks_stop(proc, path, device):
    if proc is None:
        return None
    proc.terminate()
    try:
        proc.wait(timeout=5)
    except Exception:
        proc.kill()
    sm, smax, reasons = [], [], set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    for line in Path(path).read_text().splitlines():
        f = [x.strip() for x in line.split(",")]
        if len(f) < 9 or not f[0].isdigit() or int(f[0]) != device:
            continue
        try:
            sm.append(float(f[1]))
            smax.append(float(f[2]))
        except ValueError:
            continue
        for n, v in zip(names, f[5:9]):
            if v.lower() == "active":
                reasons.add(n)
    if not sm:
        return None
    return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": float(max(smax)), "reasons": sorted(reasons),
            "samples": len(sm)}


# ------------------------------------------------------------------------- reference arm

def reduce_max(values, world):
    """Element-wise max over ranks (device timings are reported as the slowest rank's)."""
    import torch
    import torch.distributed as dist
    t = torch.tensor(values, dtype=torch.float64)
    if world > 1:
        if dist.get_backend() == "nccl":
            t = t.cuda()
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(x) for x in t.cpu()]


def reference_sample(steps, warmup):
    """Times the reference's CpuReferenceRunner on a 2-layer 31B-shaped container."""
    from g4dense_b200 import container as C
    from oracle import oracle as O
    spec = C.GEMMA4_31B_TWO_LAYERS
    with tempfile.TemporaryDirectory(dir="/tmp") as d:
        path = C.write_container(Path(d) / "b31_2layer.g4dense", spec, seed=0)
        if O.reference_available():
            model, kind = O.ReferenceModel(path), "reference"
            fwd = lambda tok, pos: model.forward(tok, pos)
        else:
            model, kind = O.RestatedModel(path, cache_dequant=False), "port"
            fwd = lambda tok, pos: model.forward(tok, pos)
        toks = np.random.default_rng(0).integers(0, 262144, warmup + steps)
        for p in range(warmup):
            fwd(int(toks[p]), p)
        t0 = time.perf_counter()
        for p in range(warmup, warmup + steps):
            fwd(int(toks[p]), p)
        dt = (time.perf_counter() - t0) / steps
    sample_bytes = 269.40e6 + 300.37e6 + 792.72e6
    t_token = dt * B31_PASS_BYTES / sample_bytes
    return {"value": 1.0 / t_token, "unit": UNIT, "cores": 1, "nproc": os.cpu_count(), "kind": kind,
            "measured_s_per_sample_position": dt, "extrapolation_factor": B31_PASS_BYTES / sample_bytes,
            "sample": f"{steps} position(s) of a 2-layer (1 sliding + 1 global) 31B-shaped container with the full "
                      f"262144x5376 embedding/LM head: {dt:.2f} s per position (measured), extrapolated to 60 layers "
                      f"by weight bytes ({B31_PASS_BYTES / sample_bytes:.2f}x) = {t_token:.1f} s/token; greedy "
                      f"autoregressive decode; the reference's CPU runner is single-threaded (src/cpu_reference.cpp "
                      f"has no threading), so 1 of the host's {os.cpu_count()} cores is used"}


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    cb = reference_sample(args.steps, args.warmup)
    # One step = one timed sample position; ms_per_step is what was measured per step (the
    # value is that time extrapolated to the 60-layer model, as cpu_baseline.sample states).
    line = {"metric": METRIC, "value": cb["value"], "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * cb["measured_s_per_sample_position"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
            "config": {"workload": "config3: 31B-shaped target greedy decode on the reference CPU path"},
            "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------- B200 arm

def run_b200(args, rank, world):
    import torch
    import torch.distributed as dist
    from g4dense_b200 import Engine
    from g4dense_b200.api import lib

    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)

    def nccl_id():
        """A fresh NCCL unique id from rank 0 for one tensor-parallel engine (None at TP = 1)."""
        if world == 1:
            return None
        buf = np.zeros(128, np.uint8)
        if rank == 0:
            lib().g4dense_nccl_unique_id(buf.ctypes.data)
        t = torch.from_numpy(buf).cuda()
        dist.broadcast(t, 0)
        return t.cpu().numpy().tobytes()

    nid = nccl_id()
    t_load = time.perf_counter()
    eng = Engine(preset="gemma4-31b", seed=0, draft_preset="gemma4-e2b", draft_seed=1, draft_k=VERIFY_WIDTH,
                 max_context=4096, tp_rank=rank, tp_size=world, nccl_id=nid, device=local)
    load_s = time.perf_counter() - t_load
    prompt = np.random.default_rng(0).integers(0, 262144, PROMPT_LEN).astype(np.uint32)

    # The target's own greedy stream, for the oracle drafter (untimed).
    eng.set_decode_options(draft_k=0)
    stream = eng.generate(prompt, GEN_LEN)
    ar = eng.stats()
    eng.set_gate(0.45, -1)  # replay runs: acceptance is set by the replay, not gated
    eng.set_decode_options(draft_k=VERIFY_WIDTH, replay=stream, mismatch_rate=MISMATCH, mismatch_seed=7)

    matches = []

    def one():
        toks = eng.generate(prompt, GEN_LEN)
        s = eng.stats()
        # Greedy speculative output must equal the greedy autoregressive stream.
        matches.append(len(toks) == GEN_LEN and toks.tolist() == stream.tolist())
        return s

    for _ in range(args.warmup):
        one()
    clk_path = f"/tmp/g4b_clocks_{os.getpid()}_{rank}.csv"
    clk = clocks_start(clk_path) if rank == 0 else None
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    stats = [one() for _ in range(args.steps)]
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    wall = time.perf_counter() - t0
    clocks = clocks_stop(clk, clk_path, local) if rank == 0 else None

    dec_ms = sum(s["decode_gpu_ms"] for s in stats)
    dec_tokens = sum(s["emitted"] - 1 for s in stats)
    emitted = sum(s["emitted"] for s in stats)
    dec_ms, wall = reduce_max([dec_ms, wall], world)
    value = dec_tokens / (dec_ms / 1000.0)
    e2e = emitted / wall

    # Acceptance sweep and natural drafter (one request each, same timing).
    sweep = {}
    for rate in (0.0, 0.25, 0.5, 1.0):
        eng.set_decode_options(draft_k=VERIFY_WIDTH, replay=stream, mismatch_rate=rate, mismatch_seed=7)
        s = one()
        sweep[str(rate)] = {"tok_s": (s["emitted"] - 1) / (s["decode_gpu_ms"] / 1000.0),
                            "acceptance": s["accepted"] / max(1.0, s["drafted"]), "rounds": int(s["rounds"])}
    eng.set_gate(0.45, 24)  # the natural drafter runs under the reference's default gate
    eng.set_decode_options(draft_k=VERIFY_WIDTH)
    eng.generate(prompt, GEN_LEN)
    s = eng.stats()
    sweep["natural_drafter"] = {"tok_s": (s["emitted"] - 1) / (s["decode_gpu_ms"] / 1000.0),
                                "acceptance": s["accepted"] / max(1.0, s["drafted"]), "gated_steps": int(s["gated_steps"])}
    ar_tok_s = (ar["emitted"] - 1) / (ar["decode_gpu_ms"] / 1000.0)

    # Roofline of the dominant kernel: the verify GEMMs of one 5-row pass.
    ms, gbytes, glaunch = eng.profile_gemms(VERIFY_WIDTH, reps=5)
    achieved = gbytes / (ms / 1000.0) / 1e9
    peak, peak_kind = peaks()
    traffic = None  # DRAM bytes per 5-row pass from the committed ncu summary (a full, TP = 1 pass)
    tf = REPO / "profiles" / "vgemm_31b_shapes_m5.md"
    if tf.exists():
        for ln in tf.read_text().splitlines():
            if ln.startswith("traffic_bytes_per_pass:"):
                traffic = int(ln.split(":")[1])
    if traffic is not None and world > 1:
        traffic = traffic // world  # one rank's shard streams 1/TP of the pass's weight bytes

    # Speculative weight-bytes bound: per round the target streams its weights once (split over
    # the ranks) and the drafter its weights K-1 times (on one GPU, serially); the tokens a round
    # yields are the accepted drafts plus one.
    rounds = max(1.0, sum(s["rounds"] for s in stats))
    tok_per_round = sum(s["emitted"] - 1 for s in stats) / rounds
    round_s = (B31_PASS_BYTES / world + (VERIFY_WIDTH - 1) * E2B_STEP_BYTES) / (peaks()[0] * 1e9)
    spec_bound = tok_per_round / round_s

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dec_ms / args.steps, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int4-g64 weights, fp32 activations/accumulation, fp16 KV", "data": "synthetic",
        "config": {"workload": "config3: 31B-shaped target + E2B-shaped drafter, greedy speculative decode k=4 "
                               "(verify width 5), oracle drafter at mismatch rate 0.25, adaptive gate off",
                   "prompt_tokens": PROMPT_LEN, "generated_tokens": GEN_LEN, "kv_context": 4096,
                   "parallelism": f"tp{world}", "weights_gb": 17.3,
                   "l2": "each verify pass streams 17.3 GB of weights, > 126 MB L2"},
        "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": sum(s["h2d_bytes"] for s in stats) / args.steps,
                "d2h_bytes_per_step": sum(s["d2h_bytes"] for s in stats) / args.steps},
        "gpu_launches": int(sum(s["launches"] for s in stats)),
        "roofline": {"bound": "hbm", "kernel": "vgemm (verify GEMM, M=5)", "achieved": achieved, "peak": peak,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak, "traffic": traffic,
                     "algorithmic_bytes_per_pass": gbytes, "launches_per_pass": glaunch,
                     "traffic_per": "pass (sum of dram__bytes_read+write over the pass's GEMM launches, ncu; "
                                    "profiles/vgemm_31b_shapes_m5.md" + (f"; scaled to one rank's 1/{world} shard"
                                                                         if world > 1 else "") + ")",
                     "ms_per_pass": ms},
        "prefill": {"prompt_tokens": PROMPT_LEN,
                    "ttft_ms": sum(s["ttft_ms"] for s in stats) / args.steps,
                    "tok_s": PROMPT_LEN / (sum(s["ttft_ms"] for s in stats) / args.steps / 1000.0),
                    "path": "tcgen05 prefill GEMM, chunks of 128 rows (target and drafter catch-up)"},
        "acceptance_sweep": sweep,
        "autoregressive_tok_s": ar_tok_s,
        "spec_stream_equals_greedy": all(matches),
        "acceptance": sum(s["accepted"] for s in stats) / max(1.0, sum(s["drafted"] for s in stats)),
        "weights_bound_tok_s_tp": peak * 1e9 / (B31_PASS_BYTES / world),
        "speculative_weights_bound": {
            "tok_s": spec_bound, "frac": value / spec_bound, "tokens_per_round": tok_per_round,
            "round_bytes": B31_PASS_BYTES / world + (VERIFY_WIDTH - 1) * E2B_STEP_BYTES,
            "how": "(31B pass bytes / TP + (K-1) x E2B step bytes) / measured HBM peak per round; tokens per round "
                   "= decoded tokens / rounds of the timed requests"},
        "load_s": load_s,
    }
    if clocks:
        line["clocks"] = clocks
    if world == 1:
        line["mtp_drafter"] = mtp_drafter(eng, prompt, stream, args)  # closes eng
        line["config1"] = config1_sweep()
    else:
        eng.close()
    if not args.no_long_context:
        line["long_context"] = long_context(args, eng_factory=lambda nid2: Engine(
            preset="gemma4-31b", seed=0, draft_preset="gemma4-e2b", draft_seed=1, draft_k=9, max_context=32768,
            kv_bf16=True, tp_rank=rank, tp_size=world, nccl_id=nid2, device=local), nccl_id=nccl_id)
    if rank != 0:
        return 0
    if world == 1 and not args.no_cpu_baseline:
        try:
            line["cpu_baseline"] = reference_sample(2, 1)
        except Exception as e:  # the baseline is reported, never required
            line["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
    print(json.dumps(line), flush=True)
    return 0


def config1_sweep(reps=10):
    """the verify GEMM alone on bf16 activations ~N(0, 1) (held as fp32 values)
    of M rows times INT4 G64 weights [N, K] with the container's distributions, fp32 output, for
    every (K, N) and M. Each cell is one launch of g4b_qmat_run (the kernel that streams the
    weights and sums its split-K slots in-kernel) timed with CUDA events on its stream, after a
    256 MiB write that evicts the 126 MB L2, so every launch reads its weights from HBM. GB/s =
    algorithmic bytes (N*K/2 packed nibbles + N*K/16 scale/bias bytes + 2*M*K bf16 activations +
    4*M*N outputs) / median launch time."""
    import torch
    from g4dense_b200 import QMat
    dev = torch.device("cuda")
    st = torch.cuda.current_stream()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1)
    peak = peaks()[0]
    cells = []
    for K, N in CONFIG1_SHAPES:
        W = torch.randint(-2 ** 31, 2 ** 31, (N, K // 8), dtype=torch.int32, device=dev, generator=gen)
        S = (torch.randn((N, K // 64), device=dev, generator=gen).abs() * 0.02).to(torch.bfloat16).view(torch.int16)
        B = (torch.randn((N, K // 64), device=dev, generator=gen) * 0.01).to(torch.bfloat16).view(torch.int16)
        q = QMat(W, S, B, stream=st)
        del W, S, B
        for M in CONFIG1_M:
            x = torch.randn((M, K), device=dev, generator=gen).to(torch.bfloat16).float()
            out = torch.empty((M, N), device=dev)
            q.prepare(x, stream=st)
            ms = []
            for r in range(reps + 2):
                flush.fill_(r & 255)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(st)
                q.run(M, out, stream=st)
                e1.record(st)
                e1.synchronize()
                if r >= 2:
                    ms.append(e0.elapsed_time(e1))
            q.check_error()
            t = float(np.median(ms))
            nbytes = N * K // 2 + N * K // 16 + 2 * M * K + 4 * M * N
            gbs = nbytes / (t / 1000.0) / 1e9
            cells.append({"M": M, "K": K, "N": N, "us": t * 1000.0, "GB_s": gbs, "frac": gbs / peak})
        q.close()
    del flush
    torch.cuda.empty_cache()
    return {"cells": cells, "peak_gbs": peak,
            "how": "one g4b_qmat_run launch per cell after a 256 MiB L2-evicting write, CUDA events, median of 10"}


def long_context(args, eng_factory, nccl_id):
    """32768-token bf16 KV filled by a 30000-token prefill, verify width 9
    (k = 8), greedy (natural drafter, gate off) and temperature-0.8 rejection sampling, at the
    run's TP size (sampled verify logits are all-gathered from the ranks' vocabulary slices)."""
    import gc
    gc.collect()
    eng = eng_factory(nccl_id())
    prompt = np.random.default_rng(4).integers(0, 262144, 30000).astype(np.uint32)
    eng.set_gate(0.45, -1)
    out = {"prompt_tokens": 30000, "kv_context": 32768, "kv": "bf16", "verify_width": 9}
    eng.generate(prompt, 32)
    s = eng.stats()
    out["greedy"] = {"tokens": int(s["emitted"]), "decode_tok_s": (s["emitted"] - 1) / (s["decode_gpu_ms"] / 1000.0),
                     "prefill_s": s["ttft_ms"] / 1000.0, "acceptance": s["accepted"] / max(1.0, s["drafted"])}
    eng.generate(prompt, 16, temperature=0.8, seed=7)
    s = eng.stats()
    out["sampled_t0.8"] = {"tokens": int(s["emitted"]),
                           "decode_tok_s": (s["emitted"] - 1) / (s["decode_gpu_ms"] / 1000.0),
                           "acceptance": s["accepted"] / max(1.0, s["drafted"])}
    out["verify_pass_ms_at_30000"] = eng.time_pass(0, 9, 3, pos=30000)
    eng.close()
    if args.gpus == 1:
        # The same pass with the full-attention layers on the cluster attention kernel instead of
        # the tensor-core long-context one (G4DENSE_ATTN_LC=0 is read when the engine loads).
        gc.collect()
        os.environ["G4DENSE_ATTN_LC"] = "0"
        try:
            ref = eng_factory(None)
            out["verify_pass_ms_at_30000_cluster_attention"] = ref.time_pass(0, 9, 3, pos=30000)
            ref.close()
        finally:
            del os.environ["G4DENSE_ATTN_LC"]
    return out


def mtp_drafter(eng, prompt, stream, args):
    """The same config-3 rounds with the MTP assistant drafter (src/mtp_runner.cpp; a synthetic
    drafter of the 31B assistant's geometry: 4 layers, hidden 1024, attending the target's last
    sliding and full-attention layers) in place of the E2B-shaped one. Same oracle drafter and
    mismatch rate, so only the drafting cost differs."""
    from g4dense_b200 import Engine
    eng.close()
    m = Engine(preset="gemma4-31b", seed=0, draft_preset="gemma4-31b-assistant", draft_seed=2,
               draft_k=VERIFY_WIDTH, max_context=4096)
    m.set_gate(0.45, -1)
    m.set_decode_options(draft_k=VERIFY_WIDTH, replay=stream, mismatch_rate=MISMATCH, mismatch_seed=7)
    ok = []
    for _ in range(max(1, args.warmup)):
        m.generate(prompt, GEN_LEN)
    ms = tok = 0.0
    for _ in range(2):
        toks = m.generate(prompt, GEN_LEN)
        ok.append(toks.tolist() == stream.tolist())
        s = m.stats()
        ms += s["decode_gpu_ms"]
        tok += s["emitted"] - 1
    step_ms = m.time_pass(2, 1, reps=20, pos=PROMPT_LEN + GEN_LEN)
    m.close()
    return {"tok_s": tok / (ms / 1000.0), "step_ms": step_ms, "spec_stream_equals_greedy": all(ok),
            "workload": "config-3 rounds (k=4, mismatch 0.25) with the MTP assistant drafter instead of E2B"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-long-context", action="store_true", help="skip BASELINE config 4 (about a minute)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl" if args.impl == "b200" else "gloo", timeout=datetime.timedelta(seconds=600))
    try:
        if args.impl == "reference":
            return run_reference(args, rank, world)
        return run_b200(args, rank, world)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
