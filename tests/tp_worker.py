"""One rank of a tensor-parallel decode, run as its own process by
tests/test_gpu_tp.py (and usable by hand):

    python tests/tp_worker.py RANK WORLD PORT CONFIG LAYERS MAX_SEQ OUT.npz

Creates rank RANK of a WORLD-GPU decoder over the synthetic CONFIG model
(LAYERS, MAX_SEQ: 0 = the config's own), or over a packed model when CONFIG is
blob:<path>, exchanges the buffer handles through a
gloo process group on 127.0.0.1:PORT, then makes the same calls on every rank:
one greedy generation, then a few steps with logits. Writes ids and this rank's
logit rows to OUT.npz.
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


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
