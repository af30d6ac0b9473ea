"""Tensor parallelism: WORLD processes, one GPU each (tests/tp_worker.py), against
one GPU over the same synthetic weights; the prompt goes through the batched
(tensor-core) prefill on both sides. Every rank computes exactly its rows of
the one-GPU step, so greedy ids and each rank's logit rows must be bit-identical.
Needs WORLD GPUs; skipped otherwise."""
import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = Path(__file__).resolve().parent


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run_ranks(tmp_path, world, name, layers, max_seq, mode=None):
    port = str(_free_port())
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs, outs = [], []
    for r in range(world):
        out = tmp_path / f"rank{r}.npz"
        outs.append(out)
        procs.append(subprocess.Popen([sys.executable, str(HERE / "tp_worker.py"), str(r), str(world), port, name,
                                       str(layers or 0), str(max_seq or 0), str(out)] + ([mode] if mode else []),
                                      env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT))
    logs = []
    for p in procs:
        try:
            logs.append(p.communicate(timeout=600)[0].decode(errors="replace"))
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            raise
    for p, log in zip(procs, logs):
        assert p.returncode == 0, log[-3000:]
    return [np.load(o) for o in outs]


@pytest.mark.parametrize("world,name,layers,max_seq", [
    (2, "tiny-llama", None, None),
    (2, "llama2-7b", 2, 160),
    (2, "tinyllama-1.1b", 2, 256),
])
def test_tensor_parallel_matches_one_gpu(pkg, tmp_path, world, name, layers, max_seq):
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    res = _run_ranks(tmp_path, world, name, layers, max_seq)
    plan = pkg.synth.config_plan(name, n_layers=layers, max_seq=max_seq)
    one = pkg.runtime.Decoder.synthetic(plan, seed=0)
    prompt = [int(t) for t in np.random.default_rng(5).integers(0, plan["vocab"], 12)]
    ids = one.generate(prompt, 20)
    one.reset()
    logits = [one.step(t, want_logits=True)[1] for t in prompt[:6]]
    assert one.query("prefill_batched") == 1
    one.close()
    _check(res, ids, logits, plan, world, 1)


def _check(res, ids, logits, plan, world, pf):
    rows = plan["vocab"] // world
    for r, got in enumerate(res):
        assert int(got["tk"][0]) == 1
        assert int(got["pf"][0]) == pf           # the same prefill path as one GPU
        assert got["ids"].tolist() == list(ids), f"rank {r}"
        ref = np.stack([lg[r * rows:(r + 1) * rows] for lg in logits])
        assert np.array_equal(got["logits"].view(np.uint32), ref.view(np.uint32)), f"rank {r}"


def test_tensor_parallel_from_a_packed_blob(pkg, tmp_path):
    """b2_create_tp: every rank slices its rows out of one packed checkpoint."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from conftest import GOLDEN
    d = GOLDEN / "cfgT"
    out = tmp_path / "m"
    assert pkg.pack.main(["--checkpoint", str(d / "model.safetensors"), "--arch", str(d / "arch.json"),
                          "--quantize", "int8", "--int8-attention", "--tp", "2", "--out", str(out)]) == 0
    blob = out.with_suffix(".b2blob")
    res = _run_ranks(tmp_path, 2, f"blob:{blob}", None, None)
    plan, _ = pkg.blob.read_blob(blob)
    one = pkg.runtime.Decoder(blob)
    prompt = [int(t) for t in np.random.default_rng(5).integers(0, plan["vocab"], 12)]
    ids = one.generate(prompt, 20)
    one.reset()
    logits = [one.step(t, want_logits=True)[1] for t in prompt[:6]]
    pf = one.query("prefill_batched")
    one.close()
    _check(res, ids, logits, plan, 2, pf)


@pytest.mark.parametrize("world,name,layers,max_seq", [
    (2, "llama2-7b", 2, 160),
    (2, "tinyllama-1.1b", 2, 200),
])
def test_tensor_parallel_batched_decode_matches_one_gpu(pkg, tmp_path, world, name, layers, max_seq):
    """Batched decode over WORLD ranks (each its rows of every GEMM, its heads, its
    vocabulary rows mirrored to every rank) equals the one-GPU batched decode bit for
    bit: ids of every call and the whole logits on every rank."""
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    sys.path.insert(0, str(HERE))
    from tp_worker import batched_calls
    res = _run_ranks(tmp_path, world, name, layers, max_seq, mode="batch")
    plan = pkg.synth.config_plan(name, n_layers=layers, max_seq=max_seq)
    one = pkg.runtime.Decoder.synthetic(plan, seed=0)
    ref = batched_calls(one, plan)
    one.close()
    for r, got in enumerate(res):
        for k in ("ids", "rec", "gen"):
            assert np.array_equal(got[k], ref[k]), (r, k)
        assert np.array_equal(got["logits"].view(np.uint32), ref["logits"].view(np.uint32)), f"rank {r}"
