"""The CPU oracle against the reference's own fixtures (no GPU)."""
import json
import math

import numpy as np
import pytest

from conftest import EXAMPLES, GOLDEN, load_example


@pytest.mark.parametrize("name", EXAMPLES)
def test_oracle_matches_reference_example_tokens(pkg, oracle, name):
    """Greedy ids of the reference's decoder examples (PyTorch, prepare.py) — the
    reference's int8 examples require an exact match (run_test_int8.sh:44-47)."""
    plan, tensors, prompt, max_new, expected = load_example(pkg, name)
    om = oracle.OracleModel(plan, tensors)
    assert om.generate(prompt, max_new) == expected


def test_oracle_thread_count_does_not_change_results(pkg, oracle):
    plan, tensors, prompt, max_new, _ = load_example(pkg, "cfgT")
    a = oracle.OracleModel(plan, tensors, threads=1).generate(prompt, max_new)
    b = oracle.OracleModel(plan, tensors, threads=4).generate(prompt, max_new)
    assert a == b and len(a) == max_new


def test_rope_golden_vector(oracle):
    """examples/rope_min/test_rope.ari:20-25 — d_head=4, theta=1e4, pos=1, [1,2,3,4]."""
    g = json.loads((GOLDEN / "rope_golden.json").read_text())
    tab = oracle.rope_table(g["max_seq"], g["d_head"], g["theta"])
    out = oracle.rope_apply(np.array(g["input"], np.float32), tab, g["pos"])
    assert np.max(np.abs(out.astype(np.float64) - np.array(g["expected"]))) < g["tol"]


def test_rope_edges(oracle):
    """tests/test_rope_edges.ari: pos 0 is the identity; pair norms survive rotation."""
    tab = oracle.rope_table(8, 8, 10000.0)
    v = np.array([0.3, -1.2, 2.5, 0.7, -0.1, 4.0, 1.5, -2.2], np.float32)
    assert np.max(np.abs(oracle.rope_apply(v, tab, 0) - v)) < 1e-6
    r = oracle.rope_apply(v, tab, 3)
    n0 = np.hypot(v[0::2].astype(np.float64), v[1::2])
    n1 = np.hypot(r[0::2].astype(np.float64), r[1::2])
    assert np.max(np.abs(n0 - n1)) < 1e-5


def lcg_fill(n, seed):
    """tests/test_attention_kv.ari:20-33: s = s*1103515245 + 12345 (i32), f = (s&65535)/32768 - 1."""
    s = seed
    out = []
    for _ in range(n):
        s = (s * 1103515245 + 12345) & 0xFFFFFFFF
        if s >= 1 << 31:
            s -= 1 << 32
        out.append((s & 65535) / 32768.0 - 1.0)
    return np.array(out, np.float32)


@pytest.mark.parametrize("max_seq", [4, 9])
def test_incremental_attention_matches_one_shot(oracle, max_seq):
    """tests/test_attention_kv.ari: incremental KV attention == one-shot causal
    attention (tol 1e-4), seq=4, d_in=d_head=8, LCG weights and biases. The -60
    tail of a max_seq > n cache must not leak either."""
    seq, d = 4, 8
    X = lcg_fill(seq * d, 11).reshape(seq, d)
    Wq, Wk, Wv = (lcg_fill(d * d, s).reshape(d, d) for s in (23, 31, 47))
    bq, bk, bv = (lcg_fill(d, s) for s in (53, 59, 67))
    Q = (X.astype(np.float64) @ Wq.T + bq) / math.sqrt(d)
    K = X.astype(np.float64) @ Wk.T + bk
    V = X.astype(np.float64) @ Wv.T + bv
    Kc = np.zeros((max_seq, d), np.float32)
    Vc = np.zeros((max_seq, d), np.float32)
    for t in range(seq):
        Kc[t], Vc[t] = K[t], V[t]
        out = oracle.attn_decode(Q[t].astype(np.float32), Kc, Vc, 1, 1, d, t + 1, max_seq)
        s = Q[t] @ K[: t + 1].T
        p = np.exp(s - s.max()); p /= p.sum()
        assert np.max(np.abs(out - p @ V[: t + 1])) < 1e-4


def test_kv_overflow_returns_minus_one_and_writes_nothing(pkg, oracle):
    """tests/test_kv_overflow.ari: the step past max_seq returns -1 untouched."""
    arch = pkg.synth.config_arch("tiny-llama", max_seq=2)
    plan = pkg.arch.decoder_plan(arch, int8_attention=True)
    om = oracle.OracleModel(plan, oracle.synth_tensors(plan, seed=5))
    assert om.step(3)[0] >= 0 and om.step(4)[0] >= 0
    assert om.count == 2
    r, _ = om.step(5)
    assert r == -1 and om.count == 2
    with pytest.raises(OverflowError):
        om.reset() or om.generate([1, 2], 2)


def test_kv_reset_matches_fresh_state(pkg, oracle):
    """tests/test_kv_reset.ari: after reset, a second prompt decodes like a fresh state."""
    plan, tensors, prompt, max_new, _ = load_example(pkg, "cfgT")
    a = oracle.OracleModel(plan, tensors)
    a.generate([7, 7, 7], 5)
    a.reset()
    b = oracle.OracleModel(plan, tensors)
    assert a.generate(prompt, max_new) == b.generate(prompt, max_new)


def test_greedy_sampling_cases(oracle):
    """tests/test_sampling.ari:11-25 (-> 4), first-max-wins ties, NaN never wins."""
    assert oracle.argmax([0.1, 1.4, -0.5, 0.9, 2.7, 0.3, -1.0, 1.0]) == 4
    assert oracle.argmax([1.0, 3.0, 3.0, 2.0]) == 1
    assert oracle.argmax([np.nan, 5.0, 1.0]) == 0
    assert oracle.argmax([1.0, np.nan, 5.0, 5.0]) == 2
    assert oracle.argmax([-np.inf, -np.inf]) == 0


def test_own_exp_is_accurate(oracle):
    xs = np.concatenate([np.linspace(-103, 88, 2001), [-60.0, -1e-7, 0.0, 1e-7, 0.5, -0.5]])
    for x in xs.astype(np.float32):
        ref = math.exp(float(x))
        got = float(oracle.exp_f(x))
        if ref < 1e-37:
            assert abs(got - ref) < 1e-44
        else:
            assert abs(got - ref) <= 2.5e-7 * ref, (x, got, ref)
    for x in np.linspace(-700, 700, 1401):
        ref = math.exp(x)
        assert abs(oracle.exp_d(x) - ref) <= 4e-16 * ref
    assert oracle.exp_d(800.0) == oracle.exp_d(700.0)      # reference math_exp clamp


def test_silu_gelu_match_definitions(oracle):
    xs = np.linspace(-30, 30, 601).astype(np.float32)
    silu = oracle.silu(xs).astype(np.float64)
    ref = xs / (1.0 + np.exp(-xs.astype(np.float64)))
    assert np.max(np.abs(silu - ref) / np.maximum(1e-30, np.abs(ref))) < 1.2e-7
    g = oracle.gelu(xs).astype(np.float64)
    x = xs.astype(np.float64)
    refg = 0.5 * x * (1 + np.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3)))
    assert np.max(np.abs(g - refg)) < 1e-6


def test_oracle_gemv_matches_float64(oracle):
    rng = np.random.default_rng(0)
    for m, n in [(5, 172), (64, 64), (33, 700)]:
        W = (rng.standard_normal((m, n)) * 0.02).astype(np.float32)
        q, s = oracle.quantize_rows(W)
        x = rng.standard_normal(n).astype(np.float32)
        y = oracle.gemv_i8(q, s, x)
        ref = (q.astype(np.float64) @ x.astype(np.float64)) * s
        assert np.max(np.abs(y - ref)) <= 1e-5 * np.max(np.abs(ref)) + 1e-7


def test_synthetic_weights_distribution(oracle):
    w = oracle.synth_f32(0, 1234, 256, 1024, 0.02)
    assert abs(float(w.mean())) < 5e-4 and abs(float(w.std()) - 0.02) < 5e-4
    q, s = oracle.synth_quant(0, 1234, 256, 1024)
    q2, s2 = oracle.quantize_rows(w)
    assert np.array_equal(q, q2) and np.array_equal(s, s2)
    qs, ss = oracle.synth_quant(0, 1234, 256, 1024, rows=(10, 20), cols=(256, 512))
    assert np.array_equal(qs, q2[10:20, 256:512]) and np.array_equal(ss, s2[10:20])
