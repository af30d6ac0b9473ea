"""Sampling beyond greedy on the GPU (sampler kernel after the LM head) against
the oracle's restatement of sampling_f32.ari and the decoder loop's LCG: the same
ids for the same seed, prompt steps advancing the generator as in the reference."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SPECS = ["temperature:0.8", "temperature:1.5", "topk:20:0.9", "topk:1:1.0", "topk:0:0.7",
         "temperature:0", "topk:300:1.0"]


@pytest.mark.parametrize("name,layers,max_seq", [("tiny-llama", None, None), ("tinyllama-1.1b", 2, 96)])
@pytest.mark.parametrize("spec", SPECS)
def test_sampled_generation_matches_oracle(pkg, oracle, name, layers, max_seq, spec):
    plan = pkg.synth.config_plan(name, n_layers=layers, max_seq=max_seq)
    om = oracle.OracleModel(plan, oracle.synth_tensors(plan, seed=0), threads=8)
    dec = pkg.runtime.Decoder.synthetic(plan, seed=0)
    rng = np.random.default_rng(5)
    prompt = rng.integers(0, plan["vocab"], 6).tolist()
    for seed in (20260502, 7):
        om.reset()
        ref = om.generate_sampled(prompt, 20, spec, seed=seed)
        dec.set_sampling(spec, seed)
        assert dec.generate(prompt, 20) == ref, (spec, seed)
    dec.close()


def test_sampling_through_steps_prefill_and_eos(pkg, oracle):
    plan = pkg.synth.config_plan("tiny-llama")
    om = oracle.OracleModel(plan, oracle.synth_tensors(plan, seed=0))
    dec = pkg.runtime.Decoder.synthetic(plan, seed=0)
    prompt = [5, 9, 11, 200]
    ref = om.generate_sampled(prompt, 12, "topk:30:1.2", seed=99)
    dec.set_sampling("topk:30:1.2", 99)
    # prefill (the generator advances once per prompt step on the host) + steps
    dec.reset()
    dec.prefill(prompt[:-1])
    tok, got = prompt[-1], []
    for _ in range(12):
        tok, _ = dec.step(tok)
        got.append(tok)
    assert got == ref
    # EOS: generation stops before emitting it
    om.reset()
    eos = ref[4]
    ref_eos = om.generate_sampled(prompt, 12, "topk:30:1.2", seed=99, eos=eos)
    assert dec.generate(prompt, 12, eos=eos) == ref_eos == ref[:ref.index(eos)]
    # back to greedy
    dec.set_sampling("greedy")
    om.reset()
    assert dec.generate(prompt, 12) == om.generate(prompt, 12)
    dec.close()


def test_packed_plan_carries_the_sampler(pkg, oracle, tmp_path):
    from conftest import GOLDEN
    d = GOLDEN / "cfgT"
    assert pkg.pack.main(["--checkpoint", str(d / "model.safetensors"), "--arch", str(d / "arch.json"),
                          "--quantize", "int8", "--int8-attention", "--sample", "temperature:0.9",
                          "--rng-seed", "1234", "--out", str(tmp_path / "m")]) == 0
    plan, tensors = pkg.blob.read_blob(tmp_path / "m.b2blob")
    om = oracle.OracleModel(plan, tensors)
    ref = om.generate_sampled([1, 2, 3], 10, "temperature:0.9", seed=1234)
    dec = pkg.runtime.Decoder(tmp_path / "m.b2blob")
    assert dec.generate([1, 2, 3], 10) == ref
    dec.close()
