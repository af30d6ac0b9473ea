"""The bench-sized configurations at full depth on the GPU against the oracle:
greedy ids and logits bit-identical to the oracle's exact mode, and the logits
within the decode path's f32 tolerance (1e-3 * max|logit|) of the reference
builtin's f32 accumulation and of an f64 truth (oracle/tolerance.py).

  Llama-2-7B: all 32 layers, 8 tokens decoded at positions 512..519 over the
  oracle's synthetic KV prefix (b2_fill_kv_synthetic == b2o_state_fill_kv).
  TinyLlama-1.1B: all 22 layers, 128-token prompt, 128 generated tokens.
"""
import os

import numpy as np
import pytest

import tolerance as T

pytestmark = pytest.mark.gpu


def _gpu_logits(dec, prefix, fed, kv_fill=None):
    dec.reset()
    if kv_fill is not None:
        dec.fill_kv_synthetic(*kv_fill)
    if prefix:
        dec.prefill(prefix)
    out, ids = [], []
    for t in fed:
        tok, lg = dec.step(t, want_logits=True)
        ids.append(tok)
        out.append(lg)
    return ids, np.stack(out)


def _check(res, gpu_ids, gpu_logits, exact_logits):
    assert gpu_ids == res["ids"]
    assert np.array_equal(gpu_logits, exact_logits)
    assert res["rel_f32acc"] <= T.TOL_F32, res
    assert res["rel_f64"] <= T.TOL_F32, res
    # greedy ids may only differ from the f32-accumulate path where the top-2
    # margin is below the tolerance
    assert res["flips_f32acc"] == 0 or res["min_margin"] < T.TOL_F32, res


def test_llama2_7b_full_depth_at_positions_512(pkg, oracle):
    plan, prefix, first, new, fill = T.case(pkg, "L7")
    assert plan["n_layers"] == 32
    tensors = oracle.synth_tensors(plan, seed=0)
    res, exact = T.measure(plan, tensors, prefix, first, new, fill)
    del tensors
    dec = pkg.runtime.Decoder.synthetic(plan, seed=0)
    fed = [first] + res["ids"][:-1]
    ids, logits = _gpu_logits(dec, prefix, fed, fill)
    dec.close()
    _check(res, ids, logits, exact)


def test_tinyllama_full_config(pkg, oracle):
    plan = pkg.synth.config_plan("tinyllama-1.1b")                 # 22 layers, max_seq 2048
    rng = np.random.default_rng(1)
    prompt = rng.integers(0, plan["vocab"], 128).tolist()
    tensors = oracle.synth_tensors(plan, seed=0)
    om = oracle.OracleModel(plan, tensors, threads=os.cpu_count())
    ref = om.generate(prompt, 128)
    dec = pkg.runtime.Decoder.synthetic(plan, seed=0)
    assert dec.generate(prompt, 128) == ref
    res, exact = T.measure(plan, tensors, prompt[:-1], prompt[-1], 128)
    assert res["ids"] == ref
    ids, logits = _gpu_logits(dec, prompt[:-1], [prompt[-1]] + ref[:-1])
    dec.close()
    _check(res, ids, logits, exact)


@pytest.mark.parametrize("name", ["T", "G"])
def test_small_configs_within_tolerance(pkg, oracle, name):
    plan, prefix, first, new, fill = T.case(pkg, name)
    res, exact = T.measure(plan, oracle.synth_tensors(plan, seed=0), prefix, first, new, fill)
    dec = pkg.runtime.Decoder.synthetic(plan, seed=0)
    ids, logits = _gpu_logits(dec, prefix, [first] + res["ids"][:-1], fill)
    dec.close()
    _check(res, ids, logits, exact)
