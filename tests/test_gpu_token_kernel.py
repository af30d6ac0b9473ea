"""The persistent token kernel (one cooperative launch per step) against the
per-layer kernels and the oracle: greedy ids and logits bit-identical, across
64-key split boundaries, for every synthetic architecture."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _pair(pkg, plan, seed=0):
    """(token-kernel decoder, per-layer decoder) over the same synthetic weights."""
    old = os.environ.get("B2_TOKEN_KERNEL")
    try:
        os.environ["B2_TOKEN_KERNEL"] = "1"
        tk = pkg.runtime.Decoder.synthetic(plan, seed=seed)
        os.environ["B2_TOKEN_KERNEL"] = "0"
        pl = pkg.runtime.Decoder.synthetic(plan, seed=seed)
    finally:
        if old is None:
            del os.environ["B2_TOKEN_KERNEL"]
        else:
            os.environ["B2_TOKEN_KERNEL"] = old
    return tk, pl


@pytest.mark.parametrize("name,layers,max_seq", [
    ("tiny-llama", None, None),
    ("gpt2-small", 2, None),
    ("tinyllama-1.1b", 2, 256),
    ("llama2-7b", 2, 160),
])
def test_token_kernel_matches_per_layer_kernels_and_oracle(pkg, oracle, name, layers, max_seq):
    plan = pkg.synth.config_plan(name, n_layers=layers, max_seq=max_seq)
    tk, pl = _pair(pkg, plan)
    assert tk.query("token_kernel") == 1
    assert tk.query("kernels_per_step") == 1
    assert pl.query("token_kernel") == 0
    om = oracle.OracleModel(plan, oracle.synth_tensors(plan, seed=0), threads=8)
    rng = np.random.default_rng(7)
    n = min(plan["max_seq"], 140)            # crosses the 64- and 128-key split boundaries
    ids = rng.integers(0, plan["vocab"], n).tolist()
    for t in ids:
        r_tok, r_log = om.step(t)
        a_tok, a_log = tk.step(t, want_logits=True)
        b_tok, b_log = pl.step(t, want_logits=True)
        assert a_tok == b_tok == r_tok
        assert np.array_equal(a_log, r_log)
        assert np.array_equal(b_log, r_log)
    tk.close()
    pl.close()


def test_token_kernel_generate_and_async_decode(pkg, oracle):
    plan = pkg.synth.config_plan("llama2-7b", n_layers=2, max_seq=200)
    dec, other = _pair(pkg, plan, seed=5)
    other.close()
    assert dec.query("token_kernel") == 1
    om = oracle.OracleModel(plan, oracle.synth_tensors(plan, seed=5), threads=8)
    prompt = list(range(300, 430))
    ref = om.generate(prompt, 60)
    assert dec.generate(prompt, 60) == ref
    # rewind into the middle of the generation and decode again on the device
    dec.set_position(len(prompt), ref[0])
    dec.decode_async(59)
    dec.sync()
    assert dec.read_output(59) == ref[1:]
    dec.close()


def test_token_kernel_long_context_equals_per_layer_kernels(pkg):
    """Positions near 3000 (47 splits x 32 heads: about ten attention items per CTA,
    so each of a CTA's attention groups takes several in turn, and a ragged last
    split): the token kernel and the per-layer kernels give the same bits."""
    plan = pkg.synth.config_plan("llama2-7b", n_layers=2, max_seq=3072)
    tk, pl = _pair(pkg, plan, seed=0)
    assert tk.query("token_kernel") == 1
    outs = []
    for dec in (tk, pl):
        dec.reset()
        dec.fill_kv_synthetic(2990, seed=4)
        logs = []
        tok = 17
        for _ in range(4):
            tok, lg = dec.step(tok, want_logits=True)
            logs.append(lg)
        outs.append(logs)
        dec.close()
    for a, b in zip(*outs):
        assert np.array_equal(a, b)


def test_token_kernel_full_size_llama2_7b_equals_per_layer_kernels(pkg):
    """All 32 layers at the bench's positions: the two paths give the same bits."""
    plan = pkg.synth.config_plan("llama2-7b")
    tk, pl = _pair(pkg, plan, seed=0)
    assert tk.query("token_kernel") == 1
    prompt = list(range(1, 9))
    outs = []
    for dec in (tk, pl):
        dec.reset()
        dec.prefill(prompt[:-1])
        logs = []
        tok = prompt[-1]
        for _ in range(4):
            tok, lg = dec.step(tok, want_logits=True)
            logs.append(lg)
        outs.append(logs)
        dec.close()
    for a, b in zip(*outs):
        assert np.array_equal(a, b)


@pytest.mark.parametrize("name", ["tiny-llama", "gpt2-small"])
def test_token_kernel_tagged_words_and_grid_barriers_agree(pkg, oracle, name):
    """On one GPU the phases meet through (value, tag) words; B2_TK_TAGS=0 makes
    them meet at grid barriers instead (the tensor-parallel mode). Both give the
    oracle's bits."""
    plan = pkg.synth.config_plan(name, n_layers=2)
    old = os.environ.get("B2_TK_TAGS")
    try:
        os.environ.pop("B2_TK_TAGS", None)
        tagged = pkg.runtime.Decoder.synthetic(plan, seed=3)
        os.environ["B2_TK_TAGS"] = "0"
        barrier = pkg.runtime.Decoder.synthetic(plan, seed=3)
    finally:
        if old is None:
            os.environ.pop("B2_TK_TAGS", None)
        else:
            os.environ["B2_TK_TAGS"] = old
    assert tagged.query("token_kernel") == 1 and tagged.query("token_tags") == 1
    assert barrier.query("token_kernel") == 1 and barrier.query("token_tags") == 0
    om = oracle.OracleModel(plan, oracle.synth_tensors(plan, seed=3), threads=8)
    n = min(plan["max_seq"], 70)             # crosses a 64-key split boundary where max_seq allows
    ids = np.random.default_rng(11).integers(0, plan["vocab"], n).tolist()
    for t in ids:
        r_tok, r_log = om.step(t)
        for dec in (tagged, barrier):
            tok, log = dec.step(t, want_logits=True)
            assert tok == r_tok
            assert np.array_equal(log, r_log)
    tagged.close()
    barrier.close()
