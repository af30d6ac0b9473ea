#!/usr/bin/env python3
"""Decode benchmark: Llama-2-7B-shaped int8 model, prompt 512 + 256 greedy tokens, batch 1.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

One step = decoding the 256 new tokens after the 512-token prompt (positions
512..767) with every input already in HBM; the KV cache of the prompt is filled
once before timing and every step rewinds to position 512, so all steps do the
same work. The roofline traffic comes from profiles/token_kernel_llama2-7b.md
(a reduced-case DRAM capture scaled by the algorithmic bytes); `batched` adds the
64-sequence configuration (64 x (1024 + 128)) on the same GPU. value = generated tokens per second of that one sequence; with N > 1
GPUs (one process each, torchrun) the model is split over them (tensor
parallelism: every matrix by output rows, attention by heads), so N GPUs decode
the same batch-1 sequence faster (strong scaling). e2e = the same metric through the public C ABI call
b2_generate (prompt from pinned host memory, prefill + decode, ids back to
pinned host memory). The roofline object is the dominant kernel, the token
kernel that runs one whole decode step per launch: algorithmic bytes per token
over its average launch time; gemv_roofline is the per-launch int8 GEMV timed
alone on the model's FFN shape. `--impl reference` times the CPU restatement of
the reference decode path (oracle/) on the host cores.

Weights: random N(0, 0.02)-like synthetic weights of the Llama-2-7B architecture
(counter-based generator, identical on GPU and host); prompt ids uniform random.
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "Llama-2-7B int8 decode tok/s (b=1) at 1/2/4/8 B200; i8 GEMV % HBM peak"
CONFIG = "llama2-7b"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=("b200", "reference"), default="b200")
    p.add_argument("--config", default=CONFIG)
    p.add_argument("--layers", type=int, default=None, help="(testing only) fewer layers")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--cpu-seconds", type=float, default=15.0)
    p.add_argument("--no-batched", action="store_true", help="skip the 64-sequence batched configuration")
    return p.parse_args()


def env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def measured_peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text()), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


class Clocks:
    """nvidia-smi sampling during the timed region (median SM clock, throttle reasons)."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.tmp = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.gpu)], stdout=self.tmp, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.tmp.flush()
        rows = []
        for line in open(self.tmp.name).read().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.tmp.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}

        def num(v):
            try:
                return float(v)
            except ValueError:
                return None
        sm = [num(r[1]) for r in rows if num(r[1])]
        reasons = set()
        for r in rows:
            for name, v in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
                                "sw_power_cap"), r[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": num(rows[0][2]), "power_w_max": max(num(r[3]) or 0 for r in rows),
                "samples": len(rows), "reasons": sorted(reasons)}


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


_ORACLE = {}


def oracle_model(pkg, plan):
    """The oracle (CPU restatement of the reference decode path) over the same
    synthetic weights as the GPU (generated on the host, untimed); built once."""
    key = json.dumps(plan, sort_keys=True)
    if key not in _ORACLE:
        sys.path.insert(0, str(ROOT / "oracle"))
        import oracle as O
        t0 = time.time()
        om = O.OracleModel(plan, O.synth_tensors(plan, seed=0), threads=os.cpu_count() or 1)
        _ORACLE[key] = (O, om, time.time() - t0)
    return _ORACLE[key]


def cpu_decode(pkg, plan, n_tokens, threads, start, seconds=None, n_min=2):
    """Decode greedy tokens with the oracle in f32-accumulate mode (the reference
    builtin's arithmetic as its README describes it: 8-lane sign-extend, convert,
    FMA) over the synthetic KV prefix of `start` positions: n_tokens of them, or
    with `seconds` as many as fit (at least n_min); returns (seconds per token, ids)."""
    O, om, _ = oracle_model(pkg, plan)
    O.set_threads(threads)
    om.threads = threads
    times, ids, tok = [], [], 1
    t_end = time.time() + seconds if seconds else None
    with O.matvec_mode(O.MATVEC_F32ACC):
        om.reset()
        om.fill_kv(start, seed=1)
        for i in range(n_tokens):
            if t_end and i >= n_min and time.time() > t_end:
                break
            if om.count >= plan["max_seq"]:
                om.reset()
                om.fill_kv(start, seed=1)
            t0 = time.perf_counter()
            tok, _ = om.step(tok)
            times.append(time.perf_counter() - t0)
            ids.append(tok)
    return times, ids


def cpu_baseline(pkg, plan, seconds):
    """Reported CPU baseline: the oracle on all host cores (as many tokens as fit in
    `seconds`, at least 2) and on one core (2 tokens, how the reference's decoder
    runs: it has no threads)."""
    threads = os.cpu_count() or 1
    P = pkg.synth.CONFIGS[CONFIG]["prompt"] if plan["max_seq"] > 512 else plan["max_seq"] // 2
    _, _, setup_s = oracle_model(pkg, plan)
    times, _ = cpu_decode(pkg, plan, plan["max_seq"] - P, threads, P, seconds=seconds)
    t1, _ = cpu_decode(pkg, plan, 2, 1, P)
    return {"value": len(times) / sum(times), "unit": "tokens/s", "cores": threads, "kind": "port",
            "single_thread": {"value": len(t1) / sum(t1), "unit": "tokens/s", "cores": 1},
            "cpu": cpu_model(),
            "sample": f"{len(times)} greedy decode tokens (positions {P}..) of the same synthetic model "
                      f"over a synthetic KV prefix, int8 matvec as f32 8-lane FMA accumulation, "
                      f"{threads} host threads; single_thread: 2 tokens on 1 thread; "
                      f"host weight generation {setup_s:.1f} s untimed"}


def run_reference(args):
    """The reference arm: the oracle (CPU restatement of the reference decode path;
    the reference's own `aric` toolchain is not installable here) on the host
    cores, all threads. One step = one greedy decode token at positions 512.. of
    the Llama-2-7B workload; W untimed steps, then K timed steps."""
    rank, _, world = env_rank()
    if rank != 0:
        return 0
    pkg = importlib.import_module("aricode-ml_b200")
    plan = pkg.synth.config_plan(args.config, n_layers=args.layers)
    threads = os.cpu_count() or 1
    P = pkg.synth.CONFIGS[args.config]["prompt"]
    _, _, setup_s = oracle_model(pkg, plan)
    times, ids = cpu_decode(pkg, plan, args.warmup + args.steps, threads, P)
    timed = times[args.warmup:]
    value = len(timed) / sum(timed)
    t1, _ = cpu_decode(pkg, plan, 2, 1, P)
    cb = {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port", "cpu": cpu_model(),
          "single_thread": {"value": len(t1) / sum(t1), "unit": "tokens/s", "cores": 1},
          "sample": f"{args.steps} timed greedy decode tokens (after {args.warmup} untimed) at positions "
                    f"{P}.. over a synthetic KV prefix, int8 matvec as f32 8-lane FMA accumulation, "
                    f"{threads} host threads; single_thread: 2 tokens on 1 thread; host weight "
                    f"generation {setup_s:.1f} s untimed"}
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
            "n_gpus": args.gpus, "device": "host CPU (no GPU used)",
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000.0 * sum(timed) / len(timed), "step": "one decode token",
            "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8 x f32", "data": "synthetic",
            "config": workload_config(args, plan),
            "cpu_baseline": cb, "tokens_head": ids[:8],
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def workload_config(args, plan):
    c = pkg_configs()[args.config]
    return {"workload": f"{args.config} int8 (per-row scales) decode, prompt {c['prompt']} + "
                        f"{c['new']} greedy tokens, batch 1",
            "layers": plan["n_layers"], "d_model": plan["d_model"], "vocab": plan["vocab"],
            "prompt_tokens": c["prompt"], "decode_tokens": c["new"], "batch": 1,
            "parallelism": f"tp{args.gpus}" if args.gpus > 1 else "single",
            "l2": "weights (6.6 GB) exceed L2 (126 MB); no flush needed"}


def pkg_configs():
    return importlib.import_module("aricode-ml_b200").synth.CONFIGS


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    import torch
    rank, local_rank, world = env_rank()
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    pkg = importlib.import_module("aricode-ml_b200")
    rt = pkg.runtime
    c = pkg.synth.CONFIGS[args.config]
    plan = pkg.synth.config_plan(args.config, n_layers=args.layers)
    P, NEW = c["prompt"], c["new"]

    if world > 1:
        def exchange(handle):
            got = [None] * world
            dist.all_gather_object(got, handle)
            return got
        dec = rt.Decoder.synthetic_tp(plan, rank, world, exchange, seed=0, device=local_rank)
    else:
        dec = rt.Decoder.synthetic(plan, seed=0, device=local_rank)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    dec.set_stream(stream.cuda_stream)
    prompt = np.random.default_rng(1).integers(0, plan["vocab"], P).astype(np.int32)

    # prefill once (untimed), remember the first generated token
    dec.reset()
    t0 = time.time()
    dec.prefill(prompt[:-1].tolist())
    first, _ = dec.step(int(prompt[-1]))
    prefill_s = time.time() - t0
    prefill = time_prefill(torch, dec, prompt, stream, plan)

    def one_step():
        dec.set_position(P, first)
        dec.decode_async(NEW - 1)

    for _ in range(args.warmup):
        one_step()
    torch.cuda.synchronize()
    ids_warm = dec.read_output(NEW)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = Clocks(local_rank)
    clocks.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        one_step()
    ev1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    if dist:
        dist.barrier()
    ms = ev0.elapsed_time(ev1) / args.steps
    ids = dec.read_output(NEW)
    assert ids == ids_warm, "decode is not deterministic across steps"
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    toks = NEW - 1
    value = toks / (ms / 1000.0)
    kps = int(dec.query("kernels_per_step"))
    launches = args.steps * (toks * kps + 1)

    # ---- whole-step roofline: algorithmic bytes per token / time per token
    peaks, peak_kind = measured_peaks()
    hbm = world * float(peaks.get("hbm_gbs", 6650.0))      # every rank streams its share
    bytes_tok = sum(pkg.synth.bytes_per_token(plan, P + i) for i in range(1, NEW)) / toks
    step_gbs = bytes_tok / (ms / 1000.0 / toks) / 1e9

    # ---- dominant kernel: int8 GEMV on the FFN shape, one launch per layer's weights
    gemv = time_gemv(torch, rt, plan, stream)

    # ---- e2e through b2_generate with pinned host buffers
    e2e = time_e2e(torch, dec, prompt, NEW, stream, dist)

    out = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8 x f32",
        "data": "synthetic", "config": workload_config(args, plan),
        # dominant kernel: the decode step itself (one launch of the token kernel per
        # token when kernels_per_step == 1); algorithmic bytes = weights + KV read
        # and written, per token, over the launch's average duration
        "roofline": {"bound": "hbm", "achieved": step_gbs, "peak": hbm, "unit": "GB/s",
                     "frac": step_gbs / hbm, "traffic": profiled_traffic("token_kernel_llama2-7b"),
                     "kernel": "token_kernel (whole decode step)" if kps == 1 else "per-layer kernels",
                     "bytes_per_launch": bytes_tok, "us_per_launch": 1000.0 * ms / toks,
                     "peak_kind": f"{peak_kind} hbm_gbs" + (f" x {world} GPUs" if world > 1 else "")},
        "gemv_roofline": {"bound": "hbm", "achieved": gemv["gbs"], "peak": hbm, "unit": "GB/s",
                          "frac": gemv["gbs"] / hbm, "traffic": gemv["traffic"],
                          "kernel": gemv["kernel"] + " (per-launch GEMV alone)",
                          "bytes_per_launch": gemv["bytes"], "us_per_launch": gemv["us"]},
        "e2e": e2e, "gpu_launches": launches, "clocks": clk,
        "decode_ms_per_token": ms / toks, "prefill_s_untimed": prefill_s, "prefill": prefill,
        "tokens_head": ids[:8],
    }
    if world == 1 and not args.no_cpu_baseline:
        out["oracle_check"] = oracle_check(pkg, dec, plan, P)
        out["cpu_baseline"] = cpu_baseline(pkg, plan, args.cpu_seconds)
    if dist:
        dist.barrier()              # no rank frees its exchange buffer while a peer may still use it
    dec.close()
    if not args.no_batched and args.layers is None:
        # the batched configuration (64 sequences x (1024 + 128)) on the same GPUs; a
        # failure there (the same on every rank: the ranks' device waits are bounded)
        # is reported beside the decode figures instead of replacing them
        torch.cuda.empty_cache()
        try:
            out["batched"] = time_batched(torch, pkg, local_rank, peaks, dist=dist, rank=rank, world=world)
        except Exception as e:             # noqa: BLE001 - reported in the line
            out["batched"] = {"error": f"{type(e).__name__}: {e}"[:300]}
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(out), flush=True)
    return 0


def time_prefill(torch, dec, prompt, stream, plan, reps=3):
    """b2_prefill of the first P - 1 prompt tokens (batched on the tensor cores for
    this plan), CUDA events on the context's stream around the call."""
    toks = prompt[:-1].tolist()
    dec.reset()
    dec.prefill(toks)                                   # warm (workspace, module load)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ms = []
    for _ in range(reps):
        dec.reset()
        torch.cuda.synchronize()
        e0.record(stream)
        dec.prefill(toks)
        e1.record(stream)
        torch.cuda.synchronize()
        ms.append(e0.elapsed_time(e1))
    best = min(ms)
    # int8 tensor-core work: 4 byte planes x (every int8 matrix of the layers) per token
    macs = 0
    for b in plan["blocks"]:
        if b["type"] == "attn":
            qd, kd = b["n_heads"] * b["d_head"], b["n_kv_heads"] * b["d_head"]
            macs += plan["d_model"] * (2 * qd + 2 * kd)
        else:
            macs += 3 * plan["d_model"] * b["d_ffn"]
    ops = 2 * 4 * macs * len(toks)
    return {"tokens": len(toks), "ms": best, "tokens_per_s": len(toks) / (best / 1000.0),
            "batched": bool(dec.query("prefill_batched")), "int8_tensor_ops": ops,
            "int8_tops": ops / (best / 1000.0) / 1e12,
            "what": "b2_prefill of the prompt minus its last token (no LM head), best of 3"}


def time_batched(torch, pkg, local_rank, peaks, layers=None, dist=None, rank=0, world=1):
    """The batched configuration: 64 sequences of Llama-2-7B, each a 1024-token
    random prompt then 128 greedy tokens, on one GPU or tensor-parallel over the
    world's GPUs (each rank its rows and heads, strong scaling). Decode: the 127 steps
    after the first generated token, every sequence one token per step, timed with
    CUDA events on the device (device-resident: each step feeds its greedy ids to
    the next), the max over ranks; value = aggregate generated tokens/s. e2e:
    b2_batch_generate from host prompts (64 prefills + 128 steps), ids back to the
    host."""
    name = "llama2-7b-b64"
    c = pkg.synth.CONFIGS[name]
    plan = pkg.synth.config_plan(name, n_layers=layers)
    B, P, NEW = c["batch"], c["prompt"], c["new"]
    rng = np.random.default_rng(2)
    prompts = rng.integers(0, plan["vocab"], (B, P)).astype(np.int32)
    if world > 1:
        def exchange(handle):
            got = [None] * world
            dist.all_gather_object(got, handle)
            return got
        dec = pkg.runtime.Decoder.synthetic_tp(plan, rank, world, exchange, seed=0, device=local_rank)
    else:
        dec = pkg.runtime.Decoder.synthetic(plan, seed=0, device=local_rank)
    stream = torch.cuda.current_stream()
    dec.set_stream(stream.cuda_stream)
    dec.batch_init(B, max_steps=NEW)
    if dist:
        dist.barrier()              # every rank's caches allocated before the first exchange

    def max_over_ranks(ms):
        if dist:
            t = torch.tensor([ms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms
    t0 = time.time()
    for z in range(B):
        dec.batch_prefill(z, prompts[z, :-1].tolist())
    prefill_s = time.time() - t0
    first, _ = dec.batch_step(prompts[:, -1].tolist())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # one timed pass of the 127 decode steps (positions P .. P + 126 of every sequence)
    torch.cuda.synchronize()
    e0.record(stream)
    dec.batch_decode_async(NEW - 1)
    e1.record(stream)
    torch.cuda.synchronize()
    dec_ms = max_over_ranks(e0.elapsed_time(e1))
    rec = dec.batch_read_output(NEW)
    toks = B * (NEW - 1)
    value = toks / (dec_ms / 1000.0)
    kv_row = sum(2 * b["n_kv_heads"] * b["d_head"] * 4 for b in plan["blocks"] if b["type"] == "attn")
    w = pkg.synth.weight_bytes(plan)
    # bytes per step: weights once + every sequence's KV rows read (positions 0..pos) and one written
    per_step = [w + B * kv_row * (P + i + 2) for i in range(NEW - 1)]
    step_bytes = sum(per_step) / len(per_step)
    gbs = step_bytes / (dec_ms / 1000.0 / (NEW - 1)) / 1e9
    hbm = float(peaks.get("hbm_gbs", 6650.0)) * world
    # e2e through b2_batch_generate (host prompts in, host ids out)
    hp = torch.from_numpy(prompts).pin_memory()
    t0 = time.time()
    e0.record(stream)
    out = dec.batch_generate(hp.numpy(), NEW)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    same = bool(out[:, 0].tolist() == first and (out.T == rec[:NEW]).all())
    if dist:
        dist.barrier()              # no rank frees its exchange buffer while a peer may still use it
    dec.close()
    return {"workload": f"{name}: {B} sequences x ({P} prompt + {NEW} greedy tokens), batch decode",
            "parallelism": f"tp{world}" if world > 1 else "one GPU",
            "value": value, "unit": "tokens/s (aggregate)", "decode_steps": NEW - 1,
            "ms_per_step": dec_ms / (NEW - 1),
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                         "bytes_per_step": step_bytes,
                         "what": "weights once + every sequence's KV rows per step, over the step time"
                                 + (f" (peak: {world} GPUs)" if world > 1 else "")},
            "prefill_s": prefill_s, "prefill_tokens_per_s": B * (P - 1) / prefill_s,
            "e2e": {"value": B * NEW / (e2e_ms / 1000.0), "unit": "tokens/s", "ms_per_generate": e2e_ms,
                    "h2d_bytes_per_step": int(prompts.nbytes), "d2h_bytes_per_step": B * NEW * 4,
                    "includes": "64 batched prefills + 128 batched decode steps"},
            "generate_equals_steps": same}


def oracle_check(pkg, dec, plan, P, n=8):
    """Outside the timed region: decode n tokens on the GPU and in the oracle's exact
    mode from the same synthetic KV prefix of P positions; ids and logits must be
    bit-identical."""
    O, om, _ = oracle_model(pkg, plan)
    O.set_threads(os.cpu_count() or 1)
    om.threads = os.cpu_count() or 1
    om.reset()
    om.fill_kv(P, seed=1)
    dec.fill_kv_synthetic(P, seed=1)
    tok_g = tok_o = 1
    ids_g, ids_o, same = [], [], True
    for _ in range(n):
        tok_g, lg = dec.step(tok_g, want_logits=True)
        tok_o, lo = om.step(tok_o)
        ids_g.append(tok_g)
        ids_o.append(tok_o)
        same = same and bool(np.array_equal(lg, lo))
    ok = same and ids_g == ids_o
    assert ok, f"GPU decode differs from the oracle: {ids_g} vs {ids_o}"
    return {"ids": ids_g, "logits_bit_identical": same, "positions": f"{P}..{P + n - 1}",
            "what": "GPU vs oracle (exact mode) from the same synthetic KV prefix"}


def time_gemv(torch, rt, plan, stream, reps=3):
    """int8 GEMV alone on the FFN gate shape [d_ffn, d_model], cycling over one
    weight matrix per layer so every launch streams from HBM; all launches are
    captured in one CUDA graph and timed with CUDA events around a replay."""
    kb = importlib.import_module("aricode-ml_b200.kbench")
    blk = next(b for b in plan["blocks"] if b["type"] == "ffn")
    m, n = blk["d_ffn"], plan["d_model"]
    L = max(2, plan["n_layers"])
    Ws = [torch.randint(-128, 128, (m, n), dtype=torch.int8, device="cuda") for _ in range(L)]
    s = torch.rand(m, device="cuda") * 1e-3
    x = torch.randn(n, device="cuda")
    y = torch.empty(m, device="cuda")
    us = kb.timed(torch, lambda W, h: rt.gemv_i8(W, s, x, y=y, stream=h), Ws, reps)
    nbytes = m * n + 4 * m + 4 * n + 4 * m
    del Ws
    return {"kernel": f"gemv_i8 {m}x{n}", "us": us, "bytes": nbytes,
            "gbs": nbytes / (us * 1e-6) / 1e9, "traffic": profiled_traffic(f"gemv_i8_{m}x{n}")}


def profiled_traffic(name):
    """DRAM bytes (read + write) per launch from the committed ncu summary
    profiles/<name>.md (its traffic_bytes_per_launch line), or None."""
    f = ROOT / "profiles" / f"{name}.md"
    try:
        for line in f.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch:"):
                return int(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


def time_e2e(torch, dec, prompt, new, stream, dist=None, reps=2):
    import ctypes
    import numpy as np
    rt = importlib.import_module("aricode-ml_b200").runtime
    P = len(prompt)
    hp = torch.from_numpy(prompt).pin_memory()
    ho = torch.empty(new, dtype=torch.int32).pin_memory()
    p_ptr = ctypes.cast(hp.data_ptr(), ctypes.POINTER(ctypes.c_int32))
    o_ptr = ctypes.cast(ho.data_ptr(), ctypes.POINTER(ctypes.c_int32))
    n = ctypes.c_int(0)
    rt.check(rt.lib().b2_generate(dec._ctx, p_ptr, P, new, -1, o_ptr, ctypes.byref(n)), dec._ctx)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        rt.check(rt.lib().b2_generate(dec._ctx, p_ptr, P, new, -1, o_ptr, ctypes.byref(n)),
                 dec._ctx)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return {"value": new / (ms / 1000.0), "unit": "tokens/s",
            "h2d_bytes_per_step": 4 * P + 64, "d2h_bytes_per_step": 4 * new + 64,
            "ms_per_generate": ms,
            "includes": "prefill of the prompt (batched on the tensor cores, each rank its rows with tensor "
                        "parallelism) + 256 decode steps"}


if __name__ == "__main__":
    sys.exit(main())
