#!/usr/bin/env python3
"""Kernel micro-benchmark for the decode library: one kernel on one shape.

    python aricode-ml_b200/kbench.py gemv --m 11008 --n 4096 [--mats 4] [--reps 20]
    python aricode-ml_b200/kbench.py attn --heads 32 --kv-heads 32 --d-head 128 --keys 640
    python aricode-ml_b200/kbench.py decode --config llama2-7b --pos 512 --tokens 8
    python aricode-ml_b200/kbench.py prefill --config llama2-7b --layers 2 --tokens 511
    python aricode-ml_b200/kbench.py batch --config llama2-7b-b64 --layers 2 --steps 8

Prints one JSON line: device time per launch (CUDA events over a captured CUDA
graph of all launches, after an untimed replay), algorithmic bytes per launch and GB/s.

gemv: int8 weights [m, n] with per-row scales, cycling over `mats` distinct
weight matrices so that every launch streams its weights from HBM (pick
mats * m * n above the 126 MB L2). Algorithmic bytes = m*n (codes) + 4m (scales)
+ 4n (x) + 4m (y).

attn: split-KV decode attention over an f32 KV cache [kv_heads][max_seq][d_head]
holding `keys` valid rows, cycling over `caches` distinct caches. Algorithmic
bytes = 2 * kv_heads * keys * d_head * 4 (K and V rows) + q and out.

decode: whole decode steps (one captured graph per token) of a synthetic model
from position `pos` (KV rows below it left as allocated), `tokens` tokens after
one untimed token; reports device time per token. For launch lists under a
profiler: few launches besides the decode steps themselves.

prefill: b2_prefill of `tokens` random prompt ids (batched on the tensor cores
for Llama-family plans), `reps` times after one untimed call; reports ms per
prefill and the int8 tensor throughput (4 byte planes x every int8 matrix of the
layers x tokens x 2 ops).

batch: batched decode of `seqs` sequences (default: the config's batch) whose
caches are filled by prefills of `prompt` ids each, then `steps` device-resident
batched steps; reports ms per step and GB/s (weights once + every sequence's KV
rows per step).
"""
from __future__ import annotations

import argparse
import importlib
import json
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))


def timed(torch, fn, items, reps):
    """Device time per launch: `reps` passes over `items` captured in one CUDA graph
    (no host launch gaps), replayed once untimed and then timed with CUDA events."""
    stream = torch.cuda.current_stream()
    for it in items:
        fn(it, stream.cuda_stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        cap = torch.cuda.current_stream().cuda_stream
        for _ in range(reps):
            for it in items:
                fn(it, cap)
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    graph.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1000.0 / (reps * len(items))


def decode(torch, pkg, args):
    plan = pkg.synth.config_plan(args.config, n_layers=args.layers)
    if not 0 <= args.pos or args.pos + args.tokens + 1 > plan["max_seq"]:
        raise SystemExit("--pos + --tokens + 1 must fit max_seq")
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    dec = pkg.runtime.Decoder.synthetic(plan, seed=0)
    dec.set_stream(stream.cuda_stream)
    dec.set_position(args.pos, 1)
    dec.decode_async(1)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    dec.decode_async(args.tokens)
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / args.tokens
    nbytes = sum(pkg.synth.bytes_per_token(plan, args.pos + 2 + i) for i in range(args.tokens)) / args.tokens
    print(json.dumps({"kernel": "decode_step", "config": args.config, "layers": plan["n_layers"], "pos": args.pos,
                      "tokens": args.tokens, "kernels_per_token": int(dec.query("kernels_per_step")),
                      "us_per_token": us, "bytes_per_token": nbytes,
                      "gbs": nbytes / (us * 1e-6) / 1e9}), flush=True)
    dec.close()


def prefill(torch, pkg, args):
    import numpy as np
    plan = pkg.synth.config_plan(args.config, n_layers=args.layers)
    if args.tokens + 1 > plan["max_seq"]:
        raise SystemExit("--tokens + 1 must fit max_seq")
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    dec = pkg.runtime.Decoder.synthetic(plan, seed=0)
    dec.set_stream(stream.cuda_stream)
    ids = np.random.default_rng(1).integers(0, plan["vocab"], args.tokens).tolist()
    dec.prefill(ids)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ms = []
    for _ in range(args.reps):
        dec.reset()
        torch.cuda.synchronize()
        e0.record(stream)
        dec.prefill(ids)
        e1.record(stream)
        torch.cuda.synchronize()
        ms.append(e0.elapsed_time(e1))
    macs = sum(plan["d_model"] * (2 * b["n_heads"] * b["d_head"] + 2 * b["n_kv_heads"] * b["d_head"])
               if b["type"] == "attn" else 3 * plan["d_model"] * b["d_ffn"] for b in plan["blocks"])
    ops = 2 * 4 * macs * args.tokens
    print(json.dumps({"kernel": "prefill", "config": args.config, "layers": plan["n_layers"], "tokens": args.tokens,
                      "batched": bool(dec.query("prefill_batched")), "ms": min(ms),
                      "tokens_per_s": args.tokens / (min(ms) / 1000.0), "int8_tops": ops / (min(ms) / 1000.0) / 1e12}),
          flush=True)
    dec.close()


def batch(torch, pkg, args):
    import numpy as np
    c = pkg.synth.CONFIGS[args.config]
    plan = pkg.synth.config_plan(args.config, n_layers=args.layers)
    B = args.seqs or c.get("batch", 1)
    P = args.prompt or c["prompt"]
    if P + args.steps + 1 > plan["max_seq"]:
        raise SystemExit("--prompt + --steps + 1 must fit max_seq")
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    dec = pkg.runtime.Decoder.synthetic(plan, seed=0)
    dec.set_stream(stream.cuda_stream)
    dec.batch_init(B, max_steps=args.steps + 1)
    rng = np.random.default_rng(2)
    prompts = rng.integers(0, plan["vocab"], (B, P))
    for z in range(B):
        dec.batch_prefill(z, prompts[z, :-1].tolist())
    dec.batch_step(prompts[:, -1].tolist())
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    dec.batch_decode_async(args.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    kv_row = sum(2 * b["n_kv_heads"] * b["d_head"] * 4 for b in plan["blocks"] if b["type"] == "attn")
    nbytes = sum(pkg.synth.weight_bytes(plan) + B * kv_row * (P + i + 2) for i in range(args.steps)) / args.steps
    print(json.dumps({"kernel": "batch_step", "config": args.config, "layers": plan["n_layers"], "seqs": B,
                      "prompt": P, "steps": args.steps, "ms_per_step": ms, "tokens_per_s": B / (ms / 1000.0),
                      "bytes_per_step": nbytes, "gbs": nbytes / (ms * 1e-3) / 1e9}), flush=True)
    dec.close()


def main():
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="kernel", required=True)
    g = sub.add_parser("gemv")
    g.add_argument("--m", type=int, default=11008)
    g.add_argument("--n", type=int, default=4096)
    g.add_argument("--mats", type=int, default=4)
    g.add_argument("--reps", type=int, default=20)
    a = sub.add_parser("attn")
    a.add_argument("--heads", type=int, default=32)
    a.add_argument("--kv-heads", type=int, default=32)
    a.add_argument("--d-head", type=int, default=128)
    a.add_argument("--keys", type=int, default=640)
    a.add_argument("--max-seq", type=int, default=768)
    a.add_argument("--caches", type=int, default=8)
    a.add_argument("--reps", type=int, default=20)
    d = sub.add_parser("decode")
    d.add_argument("--config", default="llama2-7b")
    d.add_argument("--pos", type=int, default=512)
    d.add_argument("--tokens", type=int, default=8)
    d.add_argument("--layers", type=int, default=None, help="fewer layers (small profiler captures)")
    pf = sub.add_parser("prefill")
    pf.add_argument("--config", default="llama2-7b")
    pf.add_argument("--tokens", type=int, default=511)
    pf.add_argument("--layers", type=int, default=None)
    pf.add_argument("--reps", type=int, default=3)
    bt = sub.add_parser("batch")
    bt.add_argument("--config", default="llama2-7b-b64")
    bt.add_argument("--layers", type=int, default=None)
    bt.add_argument("--seqs", type=int, default=None)
    bt.add_argument("--prompt", type=int, default=None)
    bt.add_argument("--steps", type=int, default=8)
    args = ap.parse_args()

    import torch
    pkg = importlib.import_module("aricode-ml_b200")
    rt = pkg.runtime
    if args.kernel == "decode":
        return decode(torch, pkg, args)
    if args.kernel == "prefill":
        return prefill(torch, pkg, args)
    if args.kernel == "batch":
        return batch(torch, pkg, args)
    torch.cuda.set_stream(torch.cuda.Stream())
    gen = torch.Generator(device="cuda").manual_seed(0)

    if args.kernel == "gemv":
        m, n = args.m, args.n
        Ws = [torch.randint(-128, 128, (m, n), dtype=torch.int8, device="cuda", generator=gen)
              for _ in range(args.mats)]
        s = torch.rand(m, device="cuda", generator=gen) * 1e-3
        x = torch.randn(n, device="cuda", generator=gen)
        y = torch.empty(m, device="cuda")
        us = timed(torch, lambda W, h: rt.gemv_i8(W, s, x, y=y, stream=h), Ws, args.reps)
        nbytes = m * n + 4 * m + 4 * n + 4 * m
        out = {"kernel": "gemv_i8", "m": m, "n": n, "mats": args.mats}
    else:
        H, KVH, dh, nk, S = args.heads, args.kv_heads, args.d_head, args.keys, args.max_seq
        if nk > S:
            raise SystemExit("--keys must not exceed --max-seq")
        caches = [(torch.randn(KVH, S, dh, device="cuda", generator=gen),
                   torch.randn(KVH, S, dh, device="cuda", generator=gen)) for _ in range(args.caches)]
        q = torch.randn(H * dh, device="cuda", generator=gen) * dh ** -0.5
        ws = torch.zeros(rt.attn_workspace_bytes(H, KVH, dh, S), dtype=torch.uint8, device="cuda")
        out_t = torch.empty(H * dh, device="cuda")
        us = timed(torch, lambda kv, h: rt.attn_decode(q, kv[0], kv[1], H, KVH, dh, nk, S,
                                                       workspace=ws, out=out_t, stream=h),
                   caches, args.reps)
        nbytes = 2 * KVH * nk * dh * 4 + 2 * H * dh * 4
        out = {"kernel": "attn_decode", "heads": H, "kv_heads": KVH, "d_head": dh, "keys": nk}
    out.update({"us_per_launch": us, "bytes_per_launch": nbytes, "gbs": nbytes / (us * 1e-6) / 1e9})
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
