"""``--target b200`` packer: state_dict/safetensors + arch JSON -> weight blob + launch plan.

Drop-in for the decoder path of the reference packer ``tools/aricode_pack.py``:
the CLI keeps the reference's flags (parse_args, aricode_pack.py:2474-2600),
the state-dict key resolution with its HF fallbacks and ``--keys`` template
(aricode_pack.py:2807-3234), and the per-row int8 quantiser
(aricode_pack.py:3356-3379). Instead of emitting ``.ari`` source for the
external ``aric`` compiler it writes ``<out>.b2blob`` (see blob.py) and
``<out>.plan.json`` for the CUDA runtime. ``--emit-staging`` additionally writes
the reference's per-tensor staging files (``<out>_<W>.i8``,
``<out>_<W>_scales.f32``, ``<out>_<b>.f32``) so they can be byte-compared with
the reference packer's output.

Example::

    python -m aricode-ml_b200.pack --checkpoint synth.pt --arch arch.json \
        --keys "fc{idx_plus_1}.{kind}" --quantize int8 --int8-attention \
        --target b200 --out model
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np

from . import arch as A
from .blob import write_blob


class PackError(SystemExit):
    """Pack-time validation failure (the reference raises SystemExit too)."""


# --------------------------------------------------------------------------- loading
def load_state_dict(path):
    """.pt/.pth via torch.load(weights_only=True); .safetensors via safetensors
    (aricode_pack.py:82-112)."""
    p = Path(path)
    suffix = p.suffix.lower()
    if suffix in (".pt", ".pth"):
        import torch
        sd = torch.load(str(p), map_location="cpu", weights_only=True)
        if hasattr(sd, "state_dict"):
            sd = sd.state_dict()
        return sd
    if suffix == ".safetensors":
        from safetensors.torch import load_file
        return load_file(str(p))
    raise PackError(f"cannot load a checkpoint with suffix '{suffix}': give a .pt, .pth or "
                    ".safetensors file")


def _f32(t):
    """tensor -> float32 numpy (bf16/f16 checkpoints are upcast first)."""
    if isinstance(t, np.ndarray):
        return np.ascontiguousarray(t, dtype=np.float32)
    return t.detach().float().cpu().numpy()


def expand_keys(template):
    def keys(idx, kind):
        return template.format(idx=idx, idx_plus_1=idx + 1, kind=kind)
    return keys


def _first(sd, candidates):
    for k in candidates:
        if k in sd:
            return k
    return None


# ------------------------------------------------------------------- key candidates
# The candidate lists below are the reference resolver's, in its order
# (first hit wins), so a checkpoint keyed for the reference resolves identically.
def _mha_candidates(idx, hf, dbert):
    return [f"{hf}.weight", f"attn.{hf}.weight", f"attention.{hf}.weight",
            f"layers.{idx}.attn.{hf}.weight", f"layers.{idx}.{hf}.weight",
            f"model.layers.{idx}.self_attn.{hf}.weight",
            f"transformer.layer.{idx}.attention.{dbert}.weight",
            f"layer.{idx}.attention.{dbert}.weight"]


def _gqa_candidates(idx, proj):
    hf = "o_proj" if proj == "o" else f"{proj}_proj"
    return [f"model.layers.{idx}.self_attn.{hf}.weight",
            f"layers.{idx}.self_attn.{hf}.weight",
            f"transformer.h.{idx}.self_attn.{hf}.weight",
            f"gqa{idx}.{proj}.weight"]


def _layernorm_candidates(idx):
    if idx == 0:
        return ["embeddings.LayerNorm.weight", "LayerNorm.weight", "layers.0.LayerNorm.weight",
                "layer_norm0.weight", "ln_0.weight"]
    blk, is_sa = (idx - 1) // 2, idx % 2 == 1
    which = "sa_layer_norm" if is_sa else "output_layer_norm"
    bert = (f"encoder.layer.{blk}.attention.output.LayerNorm.weight" if is_sa
            else f"encoder.layer.{blk}.output.LayerNorm.weight")
    return [f"transformer.layer.{blk}.{which}.weight", f"layer.{blk}.{which}.weight", bert,
            f"layers.{idx}.LayerNorm.weight", f"layer_norm{idx}.weight", f"ln_{idx}.weight"]


def _rmsnorm_candidates(idx):
    blk = idx // 2
    which = "input_layernorm" if idx % 2 == 0 else "post_attention_layernorm"
    return [f"model.layers.{blk}.{which}.weight", f"layers.{blk}.{which}.weight",
            "model.norm.weight", "norm.weight", f"rmsnorm{idx}.weight", f"rn_{idx}.weight"]


def _swiglu_candidates(idx, proj):
    hf = f"{proj}_proj"
    return [f"model.layers.{idx}.mlp.{hf}.weight", f"layers.{idx}.mlp.{hf}.weight",
            f"swiglu{idx}.{proj}.weight"]


_EMB_CANDIDATES = ["embeddings.word_embeddings.weight", "wte.weight", "embed.weight",
                   "tok_embeddings.weight", "embeddings.weight"]
_POS_CANDIDATES = ["embeddings.position_embeddings.weight", "position_embeddings.weight",
                   "wpe.weight", "pos_embed.weight"]


def _need_shape(what, arr, shape):
    if tuple(arr.shape) != tuple(shape):
        raise PackError(f"{what} has shape {tuple(arr.shape)}; the arch JSON implies {tuple(shape)}")


def _not_found(what, tried, sd):
    keys = sorted(sd.keys())
    sample = ", ".join(keys[:8]) + (f", ... ({len(keys)} keys)" if len(keys) > 8 else "")
    raise PackError(f"{what} not found in the checkpoint (looked for {', '.join(tried[:4])}"
                    f"{', ...' if len(tried) > 4 else ''}); checkpoint keys: {sample}")


def resolve(arch, sd, keys_template="fc{idx_plus_1}.{kind}"):
    """Arch + state dict -> list of (kind, idx, suffix, W f32, b f32 or None)."""
    keys = expand_keys(keys_template)
    out = []
    for kind, idx, args in A.arch_walk(arch):
        if idx is None:
            continue
        if kind == "linear":
            in_f, out_f = args
            wk, bk = keys(idx, "weight"), keys(idx, "bias")
            if wk not in sd or bk not in sd:
                _not_found(f"weight and bias of linear op {idx} (--keys {keys_template!r})", [wk, bk], sd)
            W, b = _f32(sd[wk]), _f32(sd[bk])
            _need_shape(f"linear op {idx} weight '{wk}'", W, (out_f, in_f))
            _need_shape(f"linear op {idx} bias '{bk}'", b, (out_f,))
            out.append((kind, idx, "", W, b))
        elif kind == "multi_head_attention_kv":
            _, d, _ = args
            for proj, hf, db in (("q", "q_proj", "q_lin"), ("k", "k_proj", "k_lin"),
                                 ("v", "v_proj", "v_lin"), ("o", "out_proj", "out_lin")):
                cw = _mha_candidates(idx, hf, db)
                wk = _first(sd, cw)
                bk = _first(sd, [c.replace(".weight", ".bias") for c in cw])
                if wk is None or bk is None:
                    _not_found(f"the {proj} projection (weight and bias) of attention op {idx}", cw, sd)
                W, b = _f32(sd[wk]), _f32(sd[bk])
                _need_shape(f"attention op {idx} {proj} weight '{wk}'", W, (d, d))
                _need_shape(f"attention op {idx} {proj} bias '{bk}'", b, (d,))
                out.append((kind, idx, proj, W, b))
        elif kind == "multi_head_attention_gqa_kv":
            for proj, (_, shape, _) in zip("qkvo", A.tensor_specs(kind, args)):
                cw = _gqa_candidates(idx, proj)
                wk = _first(sd, cw)
                if wk is None:
                    _not_found(f"the {proj} projection weight of GQA attention op {idx}", cw, sd)
                W = _f32(sd[wk])
                _need_shape(f"GQA attention op {idx} {proj} weight '{wk}'", W, shape)
                # optional bias (attn_gqa_kv_step_f32 slices b_Q/b_K/b_V/b_O when the
                # caller binds them, attention_gqa_kv_f32.ari:209-217, :266-270; Llama
                # checkpoints have none, Qwen-style ones have q/k/v biases)
                bk = wk[: -len(".weight")] + ".bias"
                b = None
                if bk in sd:
                    b = _f32(sd[bk])
                    _need_shape(f"GQA attention op {idx} {proj} bias '{bk}'", b, (shape[0],))
                out.append((kind, idx, proj, W, b))
        elif kind == "layernorm":
            dim = args[0]
            cw = _layernorm_candidates(idx)
            wk = _first(sd, cw)
            bk = _first(sd, [c.replace(".weight", ".bias") for c in cw])
            if wk is None or bk is None:
                _not_found(f"the gain and shift of layernorm op {idx}", cw, sd)
            W, b = _f32(sd[wk]), _f32(sd[bk])
            _need_shape(f"layernorm op {idx} gain '{wk}'", W, (dim,))
            _need_shape(f"layernorm op {idx} shift '{bk}'", b, (dim,))
            out.append((kind, idx, "", W, b))
        elif kind == "rmsnorm":
            dim = args[0]
            cw = _rmsnorm_candidates(idx)
            wk = _first(sd, cw)
            if wk is None:
                _not_found(f"the gain of rmsnorm op {idx}", cw, sd)
            W = _f32(sd[wk])
            _need_shape(f"rmsnorm op {idx} gain '{wk}'", W, (dim,))
            out.append((kind, idx, "", W, None))
        elif kind == "swiglu_ffn":
            for proj, (_, shape, _) in zip(("gate", "up", "down"), A.tensor_specs(kind, args)):
                cw = _swiglu_candidates(idx, proj)
                wk = _first(sd, cw)
                if wk is None:
                    _not_found(f"the {proj} projection of SwiGLU op {idx}", cw, sd)
                W = _f32(sd[wk])
                _need_shape(f"SwiGLU op {idx} {proj} weight '{wk}'", W, shape)
                out.append((kind, idx, proj, W, None))
        elif kind == "embedding":
            vocab, d, _ = args
            cw = _EMB_CANDIDATES + [f"layers.{idx}.embed.weight"]
            wk = _first(sd, cw)
            if wk is None:
                _not_found(f"the token embedding of op {idx}", cw, sd)
            W = _f32(sd[wk])
            _need_shape(f"token embedding '{wk}'", W, (vocab, d))
            out.append((kind, idx, "", W, None))
        elif kind == "positional_embedding":
            max_pos, d, _ = args
            cw = _POS_CANDIDATES + [f"layers.{idx}.pos_embed.weight"]
            wk = _first(sd, cw)
            if wk is None:
                _not_found(f"the positional embedding of op {idx}", cw, sd)
            W = _f32(sd[wk])
            _need_shape(f"positional embedding '{wk}'", W, (max_pos, d))
            out.append((kind, idx, "", W, None))
        else:
            raise PackError(f"op {kind!r} is not part of the decoder decode path")
    return out


# ----------------------------------------------------------------------- quantiser
def quantize_rows(W):
    """Per-row symmetric int8 exactly as aricode_pack.py:3356-3379 (numpy f32):
    scale = max|row|/127, q = clip(round_half_even(W/safe), -128, 127)."""
    W = np.ascontiguousarray(W, dtype=np.float32)
    if W.size:
        abs_max_row = np.abs(W).max(axis=1)
    else:
        abs_max_row = np.zeros((0,), dtype=np.float32)
    scales = abs_max_row / 127.0
    safe = np.where(scales > 0, scales, 1.0)
    q = np.round(W / safe[:, None]).clip(-128, 127).astype(np.int8)
    return q, scales.astype(np.float32)


def quantize_rows_i4(W):
    """Per-row symmetric int4 as the reference packs --int4-linear / --int4-embedding
    (aricode_pack.py:3299-3355, numpy f32): scale = max|row| / 7, q = clip(
    round_half_even(W / safe), -8, 7), two codes per byte, the even column in the
    low nibble. Returns (packed uint8 [rows, cols / 2], scales f32 [rows])."""
    W = np.asarray(W, np.float32)
    amax = np.abs(W).max(axis=1) if W.size else np.zeros((0,), np.float32)
    scales = (amax / 7.0).astype(np.float32)
    safe = np.where(scales > 0, scales, 1.0)
    q4 = np.round(W / safe[:, None]).clip(-8, 7).astype(np.int8)
    u = (q4 & 0x0F).astype(np.uint8)
    return (u[:, 0::2] | (u[:, 1::2] << 4)).astype(np.uint8), scales


def build_tensors(arch, collected, *, quantize="int8", int8_attention=False, int4_linear=False,
                  int4_embedding=False):
    """collected (from resolve) -> {name: array} in arch order, reference names,
    with ``<W>_scales`` companions for int8 (int8 arrays) and int4 (uint8 arrays of
    packed nibbles) weights."""
    if quantize != "int8":
        raise PackError("--target b200 packs the --quantize int8 decode format; pass "
                        "--quantize int8")
    qkinds = A.quantised_kinds(int8_attention)
    tensors = {}
    for kind, idx, suffix, W, b in collected:
        wname, bname = A.tensor_names(kind, idx, suffix)
        if (int4_linear and kind == "linear") or (int4_embedding and kind == "embedding"):
            if W.shape[1] % 2:
                raise PackError(f"int4 packing needs an even row length; {kind} op {idx} has {W.shape[1]}")
            q, s = quantize_rows_i4(W)
            tensors[wname] = q
            tensors[f"{wname}_scales"] = s
        elif kind in qkinds:
            q, s = quantize_rows(W)
            tensors[wname] = q
            tensors[f"{wname}_scales"] = s
        else:
            tensors[wname] = np.ascontiguousarray(W, np.float32)
        if b is not None and b.size > 0:
            tensors[bname] = np.ascontiguousarray(b, np.float32)
    return tensors


def write_staging(out_base, tensors):
    """The reference's per-tensor staging files (``<out>_<name>.i8/.i4/.f32``)."""
    base = Path(out_base)
    written = []
    ext = {np.dtype(np.int8): "i8", np.dtype(np.uint8): "i4"}
    for name, arr in tensors.items():
        if name.endswith("_scales"):
            p = base.parent / f"{base.name}_{name}.f32"
        else:
            p = base.parent / f"{base.name}_{name}.{ext.get(arr.dtype, 'f32')}"
        arr.tofile(p)
        written.append(p)
    return written


# --------------------------------------------------------------------------- CLI
def parse_args(argv=None):
    p = argparse.ArgumentParser(description="aricode-pack (--target b200 backend)")
    p.add_argument("--checkpoint", required=True)
    p.add_argument("--arch", default=None)
    p.add_argument("--keys", default="fc{idx_plus_1}.{kind}")
    p.add_argument("--input-format", choices=("mnist", "stdin", "embedded", "stdin-tokens"),
                   default="stdin-tokens")
    p.add_argument("--max-prompt-tokens", type=int, default=512)
    p.add_argument("--input-file")
    # classifier-only flags of the reference CLI: accepted by the parser so that a
    # decoder command line parses the same, refused in main() when given
    p.add_argument("--input-images", default=None)
    p.add_argument("--input-labels", default=None)
    p.add_argument("--n-test", type=int, default=None)
    p.add_argument("--mean", type=float, default=None)
    p.add_argument("--std", type=float, default=None)
    p.add_argument("--no-argmax", action="store_true")
    p.add_argument("--max-new-tokens", type=int, default=16)
    p.add_argument("--sample", default="greedy")
    p.add_argument("--eos-token", type=int, default=None)
    p.add_argument("--rng-seed", type=int, default=20260502)
    p.add_argument("--profile", action="store_true")
    p.add_argument("--int8-attention", action="store_true")
    p.add_argument("--out", default=None)
    p.add_argument("--embed", action="store_true")
    p.add_argument("--quantize", choices=("none", "int8"), default="none")
    p.add_argument("--int4-linear", action="store_true")
    p.add_argument("--int4-embedding", action="store_true")
    p.add_argument("--infer-arch", action="store_true")
    # b200 backend
    p.add_argument("--target", choices=("aric", "b200"), default="b200",
                   help="b200: weight blob + launch plan for the CUDA runtime")
    p.add_argument("--tp", type=int, default=1,
                   help="tensor-parallel degree recorded in the plan (the blob stays whole; "
                        "each rank slices its rows at load)")
    p.add_argument("--emit-staging", action="store_true",
                   help="also write the reference's per-tensor staging files")
    return p.parse_args(argv)


def pack(arch, sd, *, keys="fc{idx_plus_1}.{kind}", quantize="int8", int8_attention=False, int4_linear=False,
         int4_embedding=False,
         out=None, max_new_tokens=16, sample="greedy", eos_token=None, rng_seed=20260502,
         tp=1, emit_staging=False, input_format="stdin-tokens", input_file=None,
         max_prompt_tokens=512):
    plan = A.decoder_plan(arch, int8_attention=int8_attention)
    collected = resolve(arch, sd, keys)
    tensors = build_tensors(arch, collected, quantize=quantize, int8_attention=int8_attention,
                            int4_linear=int4_linear, int4_embedding=int4_embedding)
    for blk in plan["blocks"]:                 # GQA biases the checkpoint provides
        if blk.get("kind") == "gqa":
            gi = blk["q"][len("Wgqaq"):]
            names = {p: f"bgqa{p}{gi}" for p in "qkvo"}
            if any(n in tensors for n in names.values()):
                blk["bias"] = {p: (n if n in tensors else None) for p, n in names.items()}
    missing = [n for n in A.plan_tensor_names(plan) if n not in tensors]
    if missing:
        raise PackError(f"internal: plan references tensors the packer did not produce: "
                        f"{missing}")
    try:
        from .runtime import parse_sample
        mode, top_k, temperature = parse_sample(sample)
    except ValueError as e:
        raise PackError(str(e)) from None
    plan["generation"] = {"max_new_tokens": max_new_tokens, "sample": sample,
                          "sample_mode": mode, "top_k": top_k, "temperature": temperature,
                          "eos_token": eos_token, "rng_seed": rng_seed & 0xFFFFFFFF,
                          "input_format": input_format, "max_prompt_tokens": max_prompt_tokens}
    if tp > 1:
        _check_tp_split(plan, tp)
    plan["tp"] = {"size": tp}
    if input_file:
        plan["generation"]["prompt_file"] = str(Path(input_file).resolve())
    if out is not None:
        base = Path(out)
        write_blob(base.with_suffix(".b2blob"), tensors, plan)
        base.with_suffix(".plan.json").write_text(json.dumps(plan, indent=1, sort_keys=True))
        if emit_staging:
            write_staging(base, tensors)
        if input_format in ("stdin-tokens", "embedded"):
            write_launcher(base)
    return plan, tensors


def _check_tp_split(plan, tp):
    """--tp N: every row split (query and KV heads, d_model, d_ffn, vocab) must divide
    by N, and the tensor-parallel path covers int8 attention and SwiGLU blocks only."""
    dims = [("d_model", plan["d_model"]), ("vocab", plan["vocab"])]
    for b in plan["blocks"]:
        if b["type"] == "attn":
            if b["dtype"] != "i8" or b.get("bias"):
                raise PackError("--tp > 1 needs --int8-attention and attention without biases")
            dims += [("n_heads", b["n_heads"]), ("n_kv_heads", b["n_kv_heads"])]
        elif b["kind"] != "swiglu":
            raise PackError("--tp > 1 covers SwiGLU feed-forward blocks only")
        else:
            dims.append(("d_ffn", b["d_ffn"]))
    bad = [f"{k}={v}" for k, v in dims if v % tp]
    if bad:
        raise PackError(f"--tp {tp} does not divide {', '.join(sorted(set(bad)))}")


def write_launcher(base):
    """<out> itself: a symlink to the stdin-tokens front end (aricode-ml_b200/b2run),
    which finds <out>.b2blob from the name it was started under. tools/run_decoder.py
    starts it like the reference's packed binary (./<name> in the blob's directory)."""
    import os
    from .build import FRONT, build
    if not FRONT.exists():
        build()
    link = Path(base)
    if link.is_symlink() or link.exists():
        link.unlink()
    os.symlink(os.path.relpath(FRONT.resolve(), link.parent.resolve()), link)
    return link


def main(argv=None):
    a = parse_args(argv)
    if a.target != "b200":
        raise PackError("this packer implements --target b200 only; use the reference packer "
                        "for aric output")
    if a.infer_arch:
        raise PackError("--infer-arch covers classifier/CNN archs, which are not part of the "
                        "decoder path")
    classifier = [f for f, v in (("--input-images", a.input_images), ("--input-labels", a.input_labels),
                                 ("--n-test", a.n_test), ("--mean", a.mean), ("--std", a.std),
                                 ("--no-argmax", a.no_argmax)) if v not in (None, False)]
    if classifier or a.input_format in ("mnist", "stdin"):
        raise PackError("--target b200 packs decoders; the classifier options "
                        f"{', '.join(classifier) or '--input-format ' + a.input_format} do not apply")
    if a.input_format == "embedded" and not a.input_file:
        raise PackError("--input-format embedded reads its prompt from --input-file; none was given")
    if a.max_prompt_tokens < 1:
        raise PackError("--max-prompt-tokens must be at least 1")
    if a.profile:
        raise PackError("--profile (per-op cycle counters in the emitted binary) is not available "
                        "with --target b200; set B2_TK_TRACE=<file> at run time for a per-phase timeline")
    if a.tp < 1:
        raise PackError("--tp must be at least 1")
    if a.arch is None or a.out is None:
        raise PackError("packing needs both --arch (the arch JSON) and --out (the output base name)")
    if a.quantize != "int8":
        # the reference forces --embed for int8; b200 packs only the int8 decode format
        raise PackError("--target b200 packs the --quantize int8 decode format; pass "
                        "--quantize int8")
    arch = json.loads(Path(a.arch).read_text())
    if not isinstance(arch, list):
        raise PackError("the --arch file must hold a JSON list of ops, each [kind, args...]")
    sd = load_state_dict(a.checkpoint)
    plan, tensors = pack(arch, sd, keys=a.keys, quantize=a.quantize,
                         int8_attention=a.int8_attention, int4_linear=a.int4_linear,
                         int4_embedding=a.int4_embedding, out=a.out,
                         max_new_tokens=a.max_new_tokens, sample=a.sample,
                         eos_token=a.eos_token, rng_seed=a.rng_seed, tp=a.tp,
                         emit_staging=a.emit_staging, input_format=a.input_format,
                         input_file=a.input_file, max_prompt_tokens=a.max_prompt_tokens)
    base = Path(a.out)
    nbytes = sum(t.nbytes for t in tensors.values())
    print(f"wrote {base.with_suffix('.b2blob')}  ({len(tensors)} tensors, {nbytes} bytes)")
    print(f"wrote {base.with_suffix('.plan.json')}  ({plan['family']}, {plan['n_layers']} "
          f"blocks, d_model={plan['d_model']}, vocab={plan['vocab']})")
    return 0


if __name__ == "__main__":
    sys.exit(main())
