"""Batched prefill on the tensor cores (tcgen05 kind::i8 over the byte planes of
the fixed-point activations, prefill.cuh) against the token-at-a-time path and
the oracle: the KV cache it leaves, and so every later logit and id, must be
bit-identical."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,n,T", [(128, 128, 1), (64, 64, 9), (300, 200, 7), (256, 4096, 100),
                                   (11008, 4096, 130), (4096, 11008, 64), (32000, 2048, 257)])
def test_tensor_core_gemm_equals_gemv_per_token(pkg, oracle, m, n, T):
    import torch
    rt = pkg.runtime
    rng = np.random.default_rng(m + n + T)
    ld = (n + 15) // 16 * 16
    W = np.zeros((m, ld), np.int8)
    W[:, :n] = rng.integers(-128, 128, (m, n), dtype=np.int8)
    s = (rng.random(m, dtype=np.float32) * 1e-2).astype(np.float32)
    X = (rng.standard_normal((T, n)) * rng.choice([1e-3, 1.0, 30.0], (T, 1))).astype(np.float32)
    Wd, sd = torch.from_numpy(W).cuda(), torch.from_numpy(s).cuda()
    Y = rt.gemm_i8(Wd, sd, torch.from_numpy(X).cuda(), n=n).cpu().numpy()
    for t in range(T):
        y = rt.gemv_i8(Wd, sd, torch.from_numpy(X[t]).cuda(), n=n).cpu().numpy()
        assert np.array_equal(Y[t], y), f"token {t}"
    ref = oracle.gemv_i8(W[:, :n], s, X[T - 1])
    assert np.array_equal(Y[T - 1], ref)


def _pair(pkg, plan, seed=0):
    old = os.environ.get("B2_PREFILL_BATCHED")
    try:
        os.environ["B2_PREFILL_BATCHED"] = "0"
        seq = pkg.runtime.Decoder.synthetic(plan, seed=seed)
        os.environ.pop("B2_PREFILL_BATCHED")
        bat = pkg.runtime.Decoder.synthetic(plan, seed=seed)
    finally:
        if old is not None:
            os.environ["B2_PREFILL_BATCHED"] = old
    return bat, seq


@pytest.mark.parametrize("name,layers,max_seq,P", [
    ("tiny-llama", None, None, 20),
    ("tinyllama-1.1b", 2, 768, 600),          # two chunks of up to 512 tokens, 64-key splits
    ("llama2-7b", 2, 768, 300),
])
def test_batched_prefill_equals_token_at_a_time(pkg, oracle, name, layers, max_seq, P):
    plan = pkg.synth.config_plan(name, n_layers=layers, max_seq=max_seq)
    bat, seq = _pair(pkg, plan)
    assert bat.query("prefill_batched") == 1 and seq.query("prefill_batched") == 0
    rng = np.random.default_rng(11)
    prompt = rng.integers(0, plan["vocab"], P).tolist()
    outs = []
    for dec in (bat, seq):
        dec.reset()
        dec.prefill(prompt[:-1])
        tok, logs = prompt[-1], []
        for _ in range(4):
            tok, lg = dec.step(tok, want_logits=True)
            logs.append(lg)
        outs.append(logs)
    for a, b in zip(*outs):
        assert np.array_equal(a, b)
    om = oracle.OracleModel(plan, oracle.synth_tensors(plan, seed=0), threads=os.cpu_count())
    ref = om.generate(prompt, 6)
    assert bat.generate(prompt, 6) == ref
    bat.close()
    seq.close()


def test_prefill_continues_mid_sequence(pkg):
    """Two batched prefills back to back (the second starts at position 37) equal
    one prefill of both parts."""
    plan = pkg.synth.config_plan("llama2-7b", n_layers=1, max_seq=256)
    a = pkg.runtime.Decoder.synthetic(plan, seed=2)
    ids = list(range(100, 190))
    a.prefill(ids[:37])
    a.prefill(ids[37:-1])
    t1, l1 = a.step(ids[-1], want_logits=True)
    a.reset()
    a.prefill(ids[:-1])
    t2, l2 = a.step(ids[-1], want_logits=True)
    assert t1 == t2 and np.array_equal(l1, l2)
    a.close()
