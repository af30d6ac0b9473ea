"""The oracle's sampler against the reference's own sampling tests
(tests/test_sampling.ari, tests/test_sampling_edges.ari) and the decoder loop's
LCG (aricode_pack.py:2291-2306). CPU only."""
import numpy as np
import pytest


def fill_distinct(n, argmax_at):
    """tests/test_sampling_edges.ari fill_distinct: 5.0 at argmax_at, i*0.1 - 1 elsewhere (f32)."""
    v = np.array([np.float32(np.float64(np.float32(i)) * 0.1 - 1.0) for i in range(n)], np.float32)
    v[argmax_at] = 5.0
    return v


def test_reference_sampling_cases(oracle):
    L = np.array([0.1, 1.4, -0.5, 0.9, 2.7, 0.3, -1.0, 1.0], np.float32)
    assert oracle.argmax(L) == 4
    f = oracle.topk_filter(L, 2)
    assert f[7] < -1000 and f[1] >= 1.3 and f[4] >= 2.6
    assert oracle.sample_temperature(np.array([0, 0, 5, 0], np.float32), 0.1, 0.5)[0] == 2


@pytest.mark.parametrize("unit", [0.001, 0.5, 0.999, 0.0])
def test_topk1_is_greedy_for_any_draw(oracle, unit):
    L = oracle.topk_filter(fill_distinct(8, 5), 1)
    assert oracle.sample_temperature(L, 1.0, np.float64(np.float32(unit)))[0] == 5


def test_topk_k_at_least_n_is_a_no_op(oracle):
    for k in (8, 108):
        L = fill_distinct(8, 3)
        assert np.array_equal(oracle.topk_filter(L, k), L)


def test_temperature_writes_softmax_in_place(oracle):
    tok, p = oracle.sample_temperature(np.array([0, 0, 5, 0], np.float32), 1.0, 0.5)
    assert abs(float(np.sum(p.astype(np.float64))) - 1.0) < 1e-4 and p[2] > 0.9


def test_non_positive_temperature_is_greedy(oracle):
    assert oracle.sample_temperature(fill_distinct(8, 5), 0.0, 0.5)[0] == 5
    assert oracle.sample_temperature(fill_distinct(8, 2), -0.5, 0.7)[0] == 2


def test_topk_zero_keeps_only_the_argmax(oracle):
    f = oracle.topk_filter(fill_distinct(8, 4), 0)
    assert f[4] == 5.0 and all(f[i] < -1000 for i in range(8) if i != 4)


def test_topk_keeps_distinct_values(oracle):
    # the K passes count distinct values: ties all survive
    L = np.array([3, 3, 2, 1, 3, 0], np.float32)
    assert np.array_equal(oracle.topk_filter(L, 2) > -1000, L >= 2)


def test_lcg_matches_the_reference_loop(oracle):
    s, seq = 20260502, []
    for _ in range(4):
        s = (s * 1103515245 + 12345) & 0xFFFFFFFF
        seq.append(s)
    got, t = [], 20260502
    for _ in range(4):
        t = oracle.lcg_next(t)
        got.append(t)
    assert got == seq


def test_sampled_generation_is_deterministic_and_seeded(pkg, oracle):
    plan = pkg.synth.config_plan("tiny-llama")
    om = oracle.OracleModel(plan, oracle.synth_tensors(plan, seed=0))
    a = om.generate_sampled([1, 2, 3], 12, "topk:20:0.9", seed=7)
    om.reset()
    b = om.generate_sampled([1, 2, 3], 12, "topk:20:0.9", seed=7)
    om.reset()
    c = om.generate_sampled([1, 2, 3], 12, "topk:20:0.9", seed=8)
    om.reset()
    g = om.generate_sampled([1, 2, 3], 12, "greedy")
    om.reset()
    assert a == b and a != c
    assert g == om.generate([1, 2, 3], 12)
