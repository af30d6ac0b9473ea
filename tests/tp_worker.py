"""One rank of a tensor-parallel decode, run as its own process by
tests/test_gpu_tp.py (and usable by hand):

    python tests/tp_worker.py RANK WORLD PORT CONFIG LAYERS MAX_SEQ OUT.npz [batch]

Creates rank RANK of a WORLD-GPU decoder over the synthetic CONFIG model
(LAYERS, MAX_SEQ: 0 = the config's own), or over a packed model when CONFIG is
blob:<path>, exchanges the buffer handles through a
gloo process group on 127.0.0.1:PORT, then makes the same calls on every rank:
one greedy generation, then a few steps with logits. Writes ids and this rank's
logit rows to OUT.npz. With `batch`: the batched decode instead (batched_calls,
also run on one GPU by the test), its ids and whole logits.
"""
import datetime
import importlib
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]


def main(argv):
    rank, world, port = int(argv[0]), int(argv[1]), argv[2]
    name, layers, max_seq, out = argv[3], int(argv[4]) or None, int(argv[5]) or None, argv[6]
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = port
    sys.path.insert(0, str(ROOT))
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    torch.cuda.set_device(rank)
    pkg = importlib.import_module("aricode-ml_b200")
    blob = name[len("blob:"):] if name.startswith("blob:") else None
    if blob:
        plan, _ = pkg.blob.read_blob(blob)
    else:
        plan = pkg.synth.config_plan(name, n_layers=layers, max_seq=max_seq)

    def exchange(handle):
        got = [None] * world
        dist.all_gather_object(got, handle)
        return got

    if blob:
        dec = pkg.runtime.Decoder.from_blob_tp(blob, rank, world, exchange, device=rank)
    else:
        dec = pkg.runtime.Decoder.synthetic_tp(plan, rank, world, exchange, seed=0, device=rank)
    if len(argv) > 7 and argv[7] == "batch":
        dist.barrier()                      # every rank set up before the first exchange
        np.savez(out, **batched_calls(dec, plan, dist.barrier))
        dist.barrier()
        dec.close()
        dist.destroy_process_group()
        return 0
    prompt = [int(t) for t in np.random.default_rng(5).integers(0, plan["vocab"], 12)]
    ids = dec.generate(prompt, 20)
    dec.reset()
    rows = plan["vocab"] // world
    logits = []
    for t in prompt[:6]:
        _, lg = dec.step(t, want_logits=True)
        logits.append(lg[rank * rows:(rank + 1) * rows])
    np.savez(out, ids=np.asarray(ids, np.int64), logits=np.stack(logits),
             tk=np.asarray([dec.query("token_kernel")]), pf=np.asarray([dec.query("prefill_batched")]))
    dist.barrier()
    dec.close()
    dist.destroy_process_group()
    return 0


def batched_calls(dec, plan, barrier=lambda: None):
    """Four sequences of different prompt lengths: batched prefills, six steps with
    logits, four device-resident steps, then b2_batch_generate over equal-length
    prompts. Returns the ids and logits."""
    B = 4
    rng = np.random.default_rng(3)
    lens = [int(x) for x in rng.integers(2, min(plan["max_seq"] // 2, 60), B)]
    prompts = [rng.integers(0, plan["vocab"], n).tolist() for n in lens]
    dec.batch_init(B, max_steps=16)
    barrier()                               # the caches are allocated on every rank
    for z, pr in enumerate(prompts):
        dec.batch_prefill(z, pr[:-1])
    toks, ids, logits = [pr[-1] for pr in prompts], [], []
    for _ in range(6):
        toks, lg = dec.batch_step(toks, want_logits=True)
        ids.append(toks)
        logits.append(lg)
    dec.batch_decode_async(4)
    rec = dec.batch_read_output(16)
    dec.batch_reset()
    gen = dec.batch_generate(rng.integers(0, plan["vocab"], (B, 20)), 8)
    return {"ids": np.asarray(ids, np.int64), "logits": np.stack(logits), "rec": rec, "gen": gen}


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
