"""How far the GPU's int8 matvec arithmetic sits from the reference's and from a
high-precision truth, measured on whole models.

TEST INFRASTRUCTURE (imported by tests/ only; ``python oracle/tolerance.py``
prints the table quoted in the design notes).

The GPU reproduces the oracle's exact mode (MATVEC_EXACT: fixed-point int8 dot,
one rounding) bit for bit, which the GPU tests assert. Here the same model is
stepped three times over one token sequence (teacher forcing: every run is fed
the exact mode's greedy ids), with the int8 matvec computed
  - exactly (the GPU's bits),
  - by f32 8-lane FMA accumulation (the reference builtin as its README describes
    it, README.md:128-131),
  - in f64 (truth for the matvec),
and the logits are compared step by step:
  rel_f32acc = max_t max|logit_exact - logit_f32acc| / max|logit_f32acc|
  rel_f64    = the same against the f64 run
  margin     = min_t (top1 - top2) / max|logit| of the f64 logits
  flips_*    = steps whose argmax differs from the exact run's.
The decode-path tolerance for f32-accumulate paths is 1e-3 * max|logit|.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import oracle as O  # noqa: E402

TOL_F32 = 1e-3


def run_logits(om, prefix, tokens, mode, kv_fill=None):
    """Logits of every step over `tokens` after feeding `prefix` (no logits) or after
    a synthetic KV fill (kv_fill = (count, seed)). Returns [len(tokens), vocab]."""
    with O.matvec_mode(mode):
        om.reset()
        if kv_fill is not None:
            om.fill_kv(*kv_fill)
        for t in prefix:
            om.step(t, want_logits=False)
        out = []
        for t in tokens:
            _, lg = om.step(t)
            out.append(lg)
    return np.stack(out)


def greedy_tokens(om, prefix, first, n, kv_fill=None):
    """The exact mode's greedy continuation: [first, id1, ..., id_{n-1}] fed tokens
    and the n ids they produce."""
    with O.matvec_mode(O.MATVEC_EXACT):
        om.reset()
        if kv_fill is not None:
            om.fill_kv(*kv_fill)
        for t in prefix:
            om.step(t, want_logits=False)
        fed, ids, tok = [], [], first
        for _ in range(n):
            fed.append(tok)
            tok, _ = om.step(tok)
            ids.append(tok)
    return fed, ids


def compare(exact, f32acc, f64):
    def rel(a, b):
        return float(max(np.max(np.abs(a[t] - b[t])) / np.max(np.abs(b[t])) for t in range(len(a))))

    def margin(lg):
        s = np.sort(lg)[::-1]
        return (s[0] - s[1]) / np.max(np.abs(lg))

    ax = exact.argmax(1)
    return {"steps": len(exact),
            "rel_f32acc": rel(exact, f32acc), "rel_f64": rel(exact, f64),
            "rel_f32acc_vs_f64": rel(f32acc, f64),
            "min_margin": float(min(margin(l) for l in f64)),
            "flips_f32acc": int(np.sum(ax != f32acc.argmax(1))),
            "flips_f64": int(np.sum(ax != f64.argmax(1)))}


def measure(plan, tensors, prefix, first, n, kv_fill=None, threads=None):
    om = O.OracleModel(plan, tensors, threads=threads or os.cpu_count() or 1)
    fed, ids = greedy_tokens(om, prefix, first, n, kv_fill)
    logs = [run_logits(om, prefix, fed, m, kv_fill) for m in (O.MATVEC_EXACT, O.MATVEC_F32ACC, O.MATVEC_F64)]
    res = compare(*logs)
    res["ids"] = ids
    return res, logs[0]


CASES = {
    # name: (config, layers, max_seq, prompt length, new tokens, kv fill)
    "T": ("tiny-llama", None, None, 8, 16, None),
    "G": ("gpt2-small", None, None, 8, 16, None),
    "TL": ("tinyllama-1.1b", None, 256, 128, 128, None),
    "L7": ("llama2-7b", None, None, 0, 8, (512, 1)),
}


def case(pkg, name):
    cfg, layers, max_seq, P, new, fill = CASES[name]
    plan = pkg.synth.config_plan(cfg, n_layers=layers, max_seq=max_seq)
    rng = np.random.default_rng(1)
    prompt = rng.integers(0, plan["vocab"], max(P, 1)).tolist()
    prefix, first = (prompt[:-1], prompt[-1]) if P else ([], prompt[0])
    return plan, prefix, first, new, fill


def main():
    import importlib
    sys.path.insert(0, str(HERE.parent))
    pkg = importlib.import_module("aricode-ml_b200")
    names = sys.argv[1:] or list(CASES)
    print("| config | steps | max rel dlogit vs f32-acc | vs f64 | f32-acc vs f64 | min top-2 margin | argmax flips (f32-acc / f64) |")
    print("|---|---|---|---|---|---|---|")
    for name in names:
        plan, prefix, first, new, fill = case(pkg, name)
        r, _ = measure(plan, O.synth_tensors(plan, seed=0), prefix, first, new, fill)
        print(f"| {name} | {r['steps']} | {r['rel_f32acc']:.2e} | {r['rel_f64']:.2e} | "
              f"{r['rel_f32acc_vs_f64']:.2e} | {r['min_margin']:.2e} | {r['flips_f32acc']} / {r['flips_f64']} |",
              flush=True)


if __name__ == "__main__":
    main()
