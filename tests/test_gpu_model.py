"""End-to-end parity through the C ABI: packed reference models and synthetic
configs decode on the GPU with greedy ids and logits identical to the oracle."""
import numpy as np
import pytest

from conftest import EXAMPLES, load_example

pytestmark = pytest.mark.gpu


def _decoder(pkg, plan, tensors, tmp_path):
    path = tmp_path / "m.b2blob"
    pkg.blob.write_blob(path, tensors, plan)
    return pkg.runtime.Decoder(path)


@pytest.mark.parametrize("name", ["cfgT"] + EXAMPLES)
def test_packed_model_tokens_and_logits(pkg, oracle, name, tmp_path):
    plan, tensors, prompt, max_new, expected = load_example(pkg, name)
    om = oracle.OracleModel(plan, tensors)
    ref = om.generate(prompt, max_new)
    if expected is not None:
        assert ref == expected
    dec = _decoder(pkg, plan, tensors, tmp_path)
    assert dec.generate(prompt, max_new) == ref
    # token-by-token with logits: bit-identical to the oracle at every position
    om.reset()
    dec.reset()
    for t in prompt + ref[:-1]:
        r_tok, r_log = om.step(t)
        g_tok, g_log = dec.step(t, want_logits=True)
        assert g_tok == r_tok
        assert np.array_equal(g_log, r_log)
    dec.close()


@pytest.mark.parametrize("name,layers,max_seq,prompt,new", [
    ("tiny-llama", None, None, 8, 16),
    ("gpt2-small", None, None, 8, 16),
    ("tinyllama-1.1b", 2, 256, 40, 24),
    ("llama2-7b", 2, 64, 8, 8),
])
def test_synthetic_config_matches_oracle(pkg, oracle, name, layers, max_seq, prompt, new):
    plan = pkg.synth.config_plan(name, n_layers=layers, max_seq=max_seq)
    rng = np.random.default_rng(1)
    ids = rng.integers(0, plan["vocab"], prompt).tolist()
    om = oracle.OracleModel(plan, oracle.synth_tensors(plan, seed=0), threads=8)
    ref = om.generate(ids, new)
    dec = pkg.runtime.Decoder.synthetic(plan, seed=0)
    assert dec.generate(ids, new) == ref
    dec.close()


def test_overflow_reset_and_eos(pkg, oracle):
    plan = pkg.synth.config_plan("tiny-llama", max_seq=10)
    dec = pkg.runtime.Decoder.synthetic(plan, seed=3)
    om = oracle.OracleModel(plan, oracle.synth_tensors(plan, seed=3))
    full = om.generate([1, 2, 3], 8)                     # 10 steps == max_seq: fits
    assert dec.generate([1, 2, 3], 8) == full
    with pytest.raises(pkg.runtime.KVOverflow):          # 11 steps: overflow is an error
        dec.generate([1, 2, 3], 9)
    assert int(dec.query("n_out")) == 8                  # ...after the ids that fit
    dec.reset()
    assert dec.generate([1, 2, 3], 8) == full            # reset == fresh state
    eos = full[3]
    got = dec.generate([1, 2, 3], 8, eos=eos)
    assert got == full[:full.index(eos)]                 # stop before emitting EOS
    dec.reset()
    for t in range(10):
        dec.step(5)
    with pytest.raises(pkg.runtime.KVOverflow):
        dec.step(5)
    dec.close()


def test_prefill_then_decode_equals_generate(pkg):
    plan = pkg.synth.config_plan("tinyllama-1.1b", n_layers=1, max_seq=128)
    dec = pkg.runtime.Decoder.synthetic(plan, seed=11)
    prompt = list(range(100, 130))
    ref = dec.generate(prompt, 20)
    dec.reset()
    dec.prefill(prompt[:-1])
    first, _ = dec.step(prompt[-1])
    dec.set_position(len(prompt), first)
    dec.decode_async(19)
    dec.sync()
    assert [first] + dec.read_output() == ref
    dec.close()


def test_bad_inputs_are_errors(pkg, tmp_path):
    plan = pkg.synth.config_plan("tiny-llama")
    dec = pkg.runtime.Decoder.synthetic(plan, seed=0)
    with pytest.raises(pkg.runtime.B2Error):
        dec.step(256)                                    # outside the vocabulary
    with pytest.raises(pkg.runtime.B2Error):
        dec.generate([-1], 2)
    dec.close()
    bad = tmp_path / "x.b2blob"
    bad.write_bytes(b"not a blob at all" * 10)
    with pytest.raises(pkg.runtime.B2Error):
        pkg.runtime.Decoder(bad)


def _with_gqa_biases(sd, projs="qkv", seed=3):
    """A copy of a Llama checkpoint with biases on the given attention projections
    (as Qwen-style checkpoints carry them)."""
    import torch
    g = torch.Generator().manual_seed(seed)
    out = dict(sd)
    for k, v in sd.items():
        for p in projs:
            hf = "o_proj" if p == "o" else f"{p}_proj"
            if k.endswith(f"self_attn.{hf}.weight"):
                out[k[: -len("weight")] + "bias"] = torch.randn(v.shape[0], generator=g) * 0.1
    return out


@pytest.mark.parametrize("name", ["tiny_llama_min", "gqa_min"])
@pytest.mark.parametrize("int8_attention", [False, True])
@pytest.mark.parametrize("projs", ["", "qkv", "qkvo"])
def test_gqa_f32_weights_and_optional_biases(pkg, oracle, name, int8_attention, projs, tmp_path):
    """GQA attention with f32 weights (no --int8-attention) and with the optional
    per-projection biases (attention_gqa_kv_f32.ari:209-217, :266-270)."""
    import json
    from conftest import GOLDEN
    d = GOLDEN / name
    man = json.loads((GOLDEN / "manifest.json").read_text())["fixtures"][name]
    arch = json.loads((d / "arch.json").read_text())
    sd = pkg.pack.load_state_dict(d / "synth.pt")
    if projs:
        sd = _with_gqa_biases(sd, projs)
    plan, tensors = pkg.pack.pack(arch, sd, int8_attention=int8_attention)
    gqa = [b for b in plan["blocks"] if b.get("kind") == "gqa"]
    assert all((b["bias"] is not None) == bool(projs) for b in gqa)
    prompt = list((d / "prompt.bin").read_bytes())
    om = oracle.OracleModel(plan, tensors)
    ref = om.generate(prompt, man["max_new"])
    if not projs:
        assert ref == man["expected_tokens"]
    dec = _decoder(pkg, plan, tensors, tmp_path)
    assert dec.generate(prompt, man["max_new"]) == ref
    om.reset()
    dec.reset()
    for t in prompt + ref[:-1]:
        r_tok, r_log = om.step(t)
        g_tok, g_log = dec.step(t, want_logits=True)
        assert g_tok == r_tok and np.array_equal(g_log, r_log)
    dec.close()
