"""One rank of the tensor-parallel parity test (launched by test_tp.py under torchrun).

argv: target container, drafter container ("-" for none), verify width, prompt (.npy of token
ids), tokens to generate, output directory, and optionally a replay stream (.npy) with its
mismatch rate and seed for the config-3 oracle drafter. G4B_TEST_SAMPLING="temperature,top_p,
top_k,seed" selects sampled decoding. Writes rank<r>.json with the greedy stream and the
per-round records. G4B_TEST_LC_LOGITS="m1,m2,..." instead feeds the prompt as forward passes of
those row counts on a bf16-KV engine (max_context 1024) and rank 0 writes logits.npz: each pass's
logits over G4B_TEST_VOCAB ids (every row of passes up to 16 rows, the last row of a prefill
chunk)."""
import json
import os
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent
sys.path[:0] = [str(REPO), str(REPO / "turbo-winfare-dense_b200")]

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main():
    target, draft, width, plen, n, out = sys.argv[1:7]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    import datetime
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    from g4dense_b200 import Engine
    from g4dense_b200.api import lib
    buf = np.zeros(128, np.uint8)
    if rank == 0:
        lib().g4dense_nccl_unique_id(buf.ctypes.data)
    t = torch.from_numpy(buf).cuda()
    dist.broadcast(t, 0)
    nid = t.cpu().numpy().tobytes()
    chunks = os.environ.get("G4B_TEST_LC_LOGITS")
    extra = {"kv_bf16": True, "max_context": 1024} if chunks else {}
    e = Engine(target=target, draft=None if draft == "-" else draft, draft_k=int(width) if draft != "-" else 0,
               tp_rank=rank, tp_size=world, nccl_id=nid, device=local, **extra)
    prompt = np.load(plen)
    if chunks:
        vocab, pos, outs = int(os.environ["G4B_TEST_VOCAB"]), 0, []
        for m in (int(x) for x in chunks.split(",")):
            outs.append(e.forward_batch(prompt[pos:pos + m], pos, vocab=vocab, all_positions=m <= 16))
            pos += m
        e.close()
        if rank == 0:
            np.savez(Path(out, "logits.npz"), *outs)
        Path(out, f"rank{rank}.json").write_text(json.dumps({"tokens": [], "rounds": []}))
        dist.barrier()
        dist.destroy_process_group()
        return
    if len(sys.argv) > 7:
        e.set_gate(0.45, -1)
        e.set_decode_options(replay=np.load(sys.argv[7]), mismatch_rate=float(sys.argv[8]),
                             mismatch_seed=int(sys.argv[9]))
    samp = os.environ.get("G4B_TEST_SAMPLING")  # "temperature,top_p,top_k,seed"
    if samp:
        t, tp, tk, seed = samp.split(",")
        toks = e.generate(prompt, int(n), temperature=float(t), top_p=float(tp), top_k=int(tk), seed=int(seed))
    else:
        toks = e.generate(prompt, int(n))
    rounds = e.rounds()
    e.close()
    Path(out, f"rank{rank}.json").write_text(json.dumps({"tokens": toks.tolist(), "rounds": rounds}))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
