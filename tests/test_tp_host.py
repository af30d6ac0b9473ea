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


def _better(va, ia, vb, ib):
    """The cross-rank argmax order of the LM-head epilogue: non-NaN beats NaN,
    larger wins, ties go to the lower vocabulary id."""
    na, nb = va != va, vb != vb
    if na != nb:
        return nb
    if not na and va != vb:
        return va > vb
    return ia < ib


def _split_rank(rank, world, port, q):
    """Each rank computes its output rows of every int8 matrix of a small model
    (whole input vector, like the GPU split) and its best logit; the gathered rows
    and the combined token must equal the one-rank results."""
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "oracle"))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import numpy as np
    import torch
    import torch.distributed as dist
    import oracle as O
    pkg = importlib.import_module("aricode-ml_b200")
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    plan = pkg.synth.config_plan("tiny-llama")
    t = O.synth_tensors(plan, seed=0)
    rng = np.random.default_rng(3)
    ok = True
    for name, dt, shape, _ in pkg.synth.tensor_specs(plan):
        if dt != "i8" or name == plan["embedding"]:
            continue
        m, n = shape
        x = rng.standard_normal(n).astype(np.float32)
        lo, hi = rank * m // world, (rank + 1) * m // world
        mine = torch.from_numpy(O.gemv_i8(t[name][lo:hi], t[name + "_scales"][lo:hi], x))
        parts = [torch.empty(m // world) for _ in range(world)]
        dist.all_gather(parts, mine)
        ok = ok and np.array_equal(torch.cat(parts).numpy(), O.gemv_i8(t[name], t[name + "_scales"], x))
    # the argmax over vocabulary rows split across the ranks
    for case in range(4):
        v = rng.standard_normal(64).astype(np.float32)
        if case == 1:
            v[[5, 40]] = v.max() + 1            # tie across the rank boundary -> lower id
        if case == 2:
            v[0] = np.nan                       # first logit NaN -> id 0 (sequential scan)
        if case == 3:
            v[[3, 50]] = np.nan                 # NaNs elsewhere never win
        lo, hi = rank * 32, (rank + 1) * 32
        bi = lo
        for i in range(lo, hi):
            if _better(v[i], i, v[bi], bi):
                bi = i
        got = [None] * world
        dist.all_gather_object(got, (float(v[bi]), bi))
        best = got[0]
        for cand in got[1:]:
            if _better(cand[0], cand[1], best[0], best[1]):
                best = cand
        tok = 0 if v[0] != v[0] else best[1]
        ok = ok and tok == O.argmax(v)
    dist.barrier()
    dist.destroy_process_group()
    q.put((rank, ok))


def test_row_split_gemv_and_argmax_equal_one_rank():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_split_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got == {0: True, 1: True}


def _batched_split_rank(rank, world, port, q):
    """The tensor-parallel batched prefill / batched decode exchange over T tokens:
    each rank computes its FFN hidden columns (gate / up rows ffn0 ..), writes them
    into every rank's copy (here an all_gather standing in for the mirrored
    stores and the flag barrier after them), then its rows of x (down rows d0 ..,
    residual added) and its vocabulary rows of the LM head the same way. Every
    rank's whole x and logits must equal the one-rank computation, and the greedy
    ids taken from the whole rows on each rank must be the one-rank ids."""
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "oracle"))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import numpy as np
    import torch
    import torch.distributed as dist
    import oracle as O
    pkg = importlib.import_module("aricode-ml_b200")
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    plan = pkg.synth.config_plan("tiny-llama")
    t = O.synth_tensors(plan, seed=0)
    ffn = next(b for b in plan["blocks"] if b["type"] == "ffn")
    d, dff, vocab = plan["d_model"], ffn["d_ffn"], plan["vocab"]
    d0, f0, v0 = rank * d // world, rank * dff // world, rank * vocab // world
    dl, fl, vl = d // world, dff // world, vocab // world

    def rows(name, lo, n, x):
        return O.gemv_i8(t[name][lo:lo + n], t[name + "_scales"][lo:lo + n], x)

    def silu_mul(g, u):                   # any elementwise map, the same on both sides
        return (g / (1.0 + np.exp(-g.astype(np.float64)))).astype(np.float32) * u

    def exchange(mine, total):            # every rank's copy of the whole row
        parts = [torch.empty(total // world) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(mine)))
        return torch.cat(parts).numpy()

    rng = np.random.default_rng(11)
    ok = True
    for tok in range(5):                  # the tokens of a chunk (or the sequences of a step)
        x = rng.standard_normal(d).astype(np.float32)
        f = exchange(silu_mul(rows(ffn["gate"], f0, fl, x), rows(ffn["up"], f0, fl, x)), dff)
        xn = exchange(x[d0:d0 + dl] + rows(ffn["down"], d0, dl, f), d)
        lg = exchange(rows(plan["lm_head"]["W"], v0, vl, xn), vocab)
        f1 = silu_mul(O.gemv_i8(t[ffn["gate"]], t[ffn["gate"] + "_scales"], x),
                      O.gemv_i8(t[ffn["up"]], t[ffn["up"] + "_scales"], x))
        x1 = x + O.gemv_i8(t[ffn["down"]], t[ffn["down"] + "_scales"], f1)
        lg1 = O.gemv_i8(t[plan["lm_head"]["W"]], t[plan["lm_head"]["W"] + "_scales"], x1)
        ok = ok and np.array_equal(f.view(np.uint32), f1.view(np.uint32))
        ok = ok and np.array_equal(xn.view(np.uint32), x1.view(np.uint32))
        ok = ok and np.array_equal(lg.view(np.uint32), lg1.view(np.uint32)) and O.argmax(lg) == O.argmax(lg1)
    dist.barrier()
    dist.destroy_process_group()
    q.put((rank, ok))


def test_batched_row_split_exchange_equals_one_rank():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_batched_split_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got == {0: True, 1: True}
