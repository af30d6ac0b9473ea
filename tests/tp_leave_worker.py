"""One rank of the "a rank leaves" failure test (tests/test_gpu_failure.py), run as
its own process; both ranks may share one GPU because only rank 0 ever launches
a step:

    python tests/tp_leave_worker.py RANK WORLD PORT DEVICE OUT.json

Both ranks create their share of a 2-rank tensor-parallel tiny Llama and connect
(exchange buffers over CUDA IPC). Rank 1 then stops taking part: it launches
nothing and only waits, alive (its buffer stays valid), until rank 0 is done.
Rank 0 runs one step; the first phase that needs rank 1's rows (the attention
output of rank 1's heads) waits for rank 1's tagged words, which never come, gives
up after its bounded wait, and the call returns B2_E_DEVICE. Rank 0 then destroys
its context cleanly and records the outcome.
"""
import datetime
import importlib
import json
import os
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def main(argv):
    rank, world, port, device, out = int(argv[0]), int(argv[1]), argv[2], int(argv[3]), argv[4]
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = port
    sys.path.insert(0, str(ROOT))
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    pkg = importlib.import_module("aricode-ml_b200")
    rt = pkg.runtime
    plan = pkg.synth.config_plan("tiny-llama")

    def exchange(handle):
        got = [None] * world
        dist.all_gather_object(got, handle)
        return got

    dec = rt.Decoder.synthetic_tp(plan, rank, world, exchange, seed=0, device=device)
    res = {"rank": rank}
    if rank == 0:
        t0 = time.time()
        try:
            dec.step(5)
            res["code"] = 0
        except rt.B2Error as e:
            res["code"] = e.code
            res["message"] = str(e)
        res["seconds"] = time.time() - t0
        res["device_err"] = dec.query("device_err")
        dec.close()
        res["destroyed"] = True
    dist.barrier()                      # rank 1 stays alive (buffer valid) until rank 0 is done
    if rank != 0:
        dec.close()
    Path(out).write_text(json.dumps(res))
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
