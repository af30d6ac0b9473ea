"""Batched decode (n_seq sequences, one token each per step, the projections as
tensor-core GEMMs over the sequences): every sequence's ids and logits must equal
decoding it alone, bit for bit, and the oracle's."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name,layers,max_seq,B", [("llama2-7b", 2, 256, 4), ("tiny-llama", None, None, 3),
                                                   ("tinyllama-1.1b", 2, 200, 5)])
def test_batched_steps_equal_single_sequences(pkg, name, layers, max_seq, B):
    plan = pkg.synth.config_plan(name, n_layers=layers, max_seq=max_seq)
    rng = np.random.default_rng(3)
    lens = [int(x) for x in rng.integers(2, min(plan["max_seq"] // 2, 90), B)]   # different positions
    prompts = [rng.integers(0, plan["vocab"], n).tolist() for n in lens]
    one = pkg.runtime.Decoder.synthetic(plan, seed=0)
    ref_ids, ref_logits = [], []
    for pr in prompts:
        one.reset()
        one.prefill(pr[:-1])
        tok, ids, logs = pr[-1], [], []
        for _ in range(6):
            tok, lg = one.step(tok, want_logits=True)
            ids.append(tok)
            logs.append(lg)
        ref_ids.append(ids)
        ref_logits.append(logs)
    one.close()
    dec = pkg.runtime.Decoder.synthetic(plan, seed=0)
    dec.batch_init(B, max_steps=16)
    for z, pr in enumerate(prompts):
        dec.batch_prefill(z, pr[:-1])
    toks = [pr[-1] for pr in prompts]
    for i in range(6):
        toks, lg = dec.batch_step(toks, want_logits=True)
        for z in range(B):
            assert toks[z] == ref_ids[z][i], (z, i)
            assert np.array_equal(lg[z], ref_logits[z][i]), (z, i)
    # the device-resident form continues the same sequences
    dec.batch_decode_async(4)
    rec = dec.batch_read_output(16)
    assert rec.shape == (10, B)
    dec.close()


def test_batch_generate_matches_oracle(pkg, oracle):
    plan = pkg.synth.config_plan("llama2-7b", n_layers=2, max_seq=160)
    B, P, new = 3, 40, 12
    rng = np.random.default_rng(9)
    prompts = rng.integers(0, plan["vocab"], (B, P))
    om = oracle.OracleModel(plan, oracle.synth_tensors(plan, seed=0), threads=os.cpu_count())
    ref = []
    for z in range(B):
        om.reset()
        ref.append(om.generate(prompts[z].tolist(), new))
    dec = pkg.runtime.Decoder.synthetic(plan, seed=0)
    dec.batch_init(B, max_steps=new)
    got = dec.batch_generate(prompts, new)
    assert got.tolist() == ref
    # b2_step with n_seq equal to the batch is the batched step; another n_seq is refused
    import ctypes as C
    rt = pkg.runtime
    dec.batch_reset()
    for z in range(B):
        dec.batch_prefill(z, prompts[z].tolist()[:-1])
    toks = (C.c_int32 * B)(*[int(prompts[z][-1]) for z in range(B)])
    nxt = (C.c_int32 * B)()
    assert rt.lib().b2_step(dec._ctx, toks, B, nxt, None) == 0
    assert list(nxt) == [r[0] for r in ref]
    assert rt.lib().b2_step(dec._ctx, toks, B + 1, nxt, None) == -7
    dec.close()


def test_batched_overflow_is_an_error(pkg):
    plan = pkg.synth.config_plan("tiny-llama", max_seq=10)
    dec = pkg.runtime.Decoder.synthetic(plan, seed=0)
    dec.batch_init(2, max_steps=32)
    dec.batch_prefill(0, list(range(1, 10)))          # sequence 0 at position 9
    dec.batch_step([1, 2])                            # position 9 is the last row
    with pytest.raises(pkg.runtime.KVOverflow):
        dec.batch_step([1, 2])
    dec.close()
