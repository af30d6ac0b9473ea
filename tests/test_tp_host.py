"""Host side of tensor parallelism on CPU: two gloo ranks (127.0.0.1) gather
their exchange-buffer handles the way bench.py and tests/tp_worker.py do, and
every rank gets the same rank-ordered concatenation; malformed exchanges are
rejected before anything reaches the library."""
import datetime
import importlib
import os
import socket
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    sys.path.insert(0, str(ROOT))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist
    rt = importlib.import_module("aricode-ml_b200.runtime")
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))

    def exchange(h):
        got = [None] * world
        dist.all_gather_object(got, h)
        return got
    mine = bytes([rank + 1]) * 64
    joined = rt.tp_gather_handles(mine, rank, world, exchange)
    dist.barrier()
    dist.destroy_process_group()
    q.put((rank, joined))


def test_handles_gathered_in_rank_order_over_gloo():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    expect = bytes([1]) * 64 + bytes([2]) * 64
    assert got[0] == expect and got[1] == expect


def test_malformed_exchanges_are_rejected(pkg):
    rt = pkg.runtime
    h = bytes(range(64))
    with pytest.raises(ValueError):
        rt.tp_gather_handles(h[:10], 0, 2, lambda x: [x, x])
    with pytest.raises(ValueError):
        rt.tp_gather_handles(h, 0, 2, lambda x: [x])                       # one rank missing
    with pytest.raises(ValueError):
        rt.tp_gather_handles(h, 0, 2, lambda x: [bytes(64), x])            # out of order
    assert rt.tp_gather_handles(h, 1, 2, lambda x: [bytes(64), x]) == bytes(64) + h
