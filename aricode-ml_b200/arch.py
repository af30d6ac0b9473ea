"""Arch-JSON op vocabulary of the reference packer, and the decoder launch plan.

The reference packer (tools/aricode_pack.py) describes a model as a JSON list of
``[kind, *args]`` entries. This module keeps that vocabulary unchanged so an
arch file written for the reference packs here too:

* per-kind weight specs       -- tensor_specs        (aricode_pack.py:841-954)
* per-kind tensor names       -- tensor_names        (aricode_pack.py:957-1006)
* per-kind running counters   -- arch_walk           (aricode_pack.py:1021-1070;
  ``multi_head_attention_kv`` shares the ``multi_head_attention`` counter)

On top of it, :func:`decoder_plan` turns a decoder arch (the archs the reference's
decoder mode packs, gen_decoder_main, aricode_pack.py:2068-2344) into the launch
plan the CUDA runtime executes: a list of pre-norm residual sub-blocks, e.g.

* llama block:  save_residual, rmsnorm, multi_head_attention_gqa_kv, add_residual,
                save_residual, rmsnorm, swiglu_ffn, add_residual
* gpt2 block:   save_residual, layernorm, multi_head_attention_kv, add_residual,
                save_residual, layernorm, linear, gelu, linear, add_residual

with ``embedding`` first (optionally followed by ``positional_embedding``) and a
final norm + ``linear`` LM head last.
"""
from __future__ import annotations

from dataclasses import dataclass

# ops carrying no weights (aricode_pack.py:402-404 plus maxpool)
PSEUDO_OPS = ("save_residual", "add_residual", "flatten", "relu", "sigmoid",
              "tanh", "softmax", "gelu", "layernorm", "rmsnorm",
              "positional_embedding")

# kind -> counter slot; multi_head_attention_kv shares multi_head_attention's
_COUNTER_SLOT = {
    "linear": "linear",
    "conv2d_3x3_p1": "conv2d_3x3_p1",
    "attention": "attention",
    "multi_head_attention": "multi_head_attention",
    "multi_head_attention_kv": "multi_head_attention",
    "multi_head_attention_gqa_kv": "multi_head_attention_gqa_kv",
    "layernorm": "layernorm",
    "rmsnorm": "rmsnorm",
    "swiglu_ffn": "swiglu_ffn",
    "embedding": "embedding",
    "positional_embedding": "positional_embedding",
}

# decode-path kinds this build executes on the GPU
DECODER_KINDS = ("embedding", "positional_embedding", "rmsnorm", "layernorm",
                 "multi_head_attention_gqa_kv", "multi_head_attention_kv",
                 "swiglu_ffn", "linear", "gelu", "save_residual", "add_residual")


class ArchError(ValueError):
    """Raised for arch lists the decoder plan cannot express."""


def arch_walk(arch):
    """Yield (kind, idx, args) with the per-kind running index (0-based,
    yielded before the bump); pseudo ops without a counter get idx None."""
    counters = {}
    for layer in arch:
        kind, *args = layer
        slot = _COUNTER_SLOT.get(kind)
        if slot is None:
            yield kind, None, list(args)
            continue
        idx = counters.get(slot, 0)
        yield kind, idx, list(args)
        counters[slot] = idx + 1


def tensor_specs(kind, args):
    """[(suffix, weight_shape, bias_len)] for one arch entry."""
    if kind == "linear":
        in_f, out_f = args
        return [("", (out_f, in_f), out_f)]
    if kind == "multi_head_attention_kv":
        max_seq, d, heads = args
        if d % heads:
            raise ArchError(f"multi_head_attention_kv: d_model ({d}) must be a multiple "
                            f"of n_heads ({heads})")
        return [(p, (d, d), d) for p in ("q", "k", "v", "o")]
    if kind == "multi_head_attention_gqa_kv":
        max_seq, d, heads, kv_heads, theta = args
        if d % heads:
            raise ArchError(f"multi_head_attention_gqa_kv: d_model ({d}) must be a "
                            f"multiple of n_heads ({heads})")
        if heads % kv_heads:
            raise ArchError(f"multi_head_attention_gqa_kv: n_heads ({heads}) must be a "
                            f"multiple of n_kv_heads ({kv_heads})")
        kv_dim = kv_heads * (d // heads)
        return [("q", (d, d), 0), ("k", (kv_dim, d), 0), ("v", (kv_dim, d), 0),
                ("o", (d, d), 0)]
    if kind == "layernorm":
        return [("", (args[0],), args[0])]
    if kind == "rmsnorm":
        return [("", (args[0],), 0)]
    if kind == "swiglu_ffn":
        d, ffn = args
        return [("gate", (ffn, d), 0), ("up", (ffn, d), 0), ("down", (d, ffn), 0)]
    if kind == "embedding":
        vocab, d, _seq = args
        return [("", (vocab, d), 0)]
    if kind == "positional_embedding":
        max_pos, d, _seq = args
        return [("", (max_pos, d), 0)]
    raise ArchError(f"no decode-path weights for {kind!r}")


def tensor_names(kind, idx, suffix=""):
    """(weight_name, bias_name) exactly as the reference stages them."""
    stem = {
        "linear": ("W", "b"),
        "multi_head_attention_kv": ("Wm", "bm"),
        "multi_head_attention": ("Wm", "bm"),
        "multi_head_attention_gqa_kv": ("Wgqa", "bgqa"),
        "layernorm": ("Wn", "bn"),
        "rmsnorm": ("Wr", "br"),
        "swiglu_ffn": ("Wsw", "bsw"),
        "embedding": ("Wemb", "bemb"),
        "positional_embedding": ("Wpos", "bpos"),
    }.get(kind)
    if stem is None:
        raise ArchError(f"tensor_names: no weights for {kind!r}")
    return f"{stem[0]}{suffix}{idx}", f"{stem[1]}{suffix}{idx}"


def weight_tensors(arch):
    """Yield (kind, idx, suffix, weight_shape, bias_len, wname, bname) in arch order."""
    for kind, idx, args in arch_walk(arch):
        if idx is None:
            continue
        for suffix, shape, nb in tensor_specs(kind, args):
            wname, bname = tensor_names(kind, idx, suffix)
            yield kind, idx, suffix, shape, nb, wname, bname


def quantised_kinds(int8_attention):
    """Kinds stored int8 per-row under --quantize int8 (aricode_pack.py:3269-3290)."""
    kinds = ["linear", "swiglu_ffn", "embedding"]
    if int8_attention:
        kinds.append("multi_head_attention_gqa_kv")
    return tuple(kinds)


def token_bytes(vocab):
    """Wire width of one token id (aricode_pack.py:483-495)."""
    return 1 if vocab <= 256 else (2 if vocab <= 65536 else 4)


@dataclass
class _Cursor:
    arch: list
    i: int = 0

    def peek(self):
        return self.arch[self.i] if self.i < len(self.arch) else None

    def take(self, kind):
        layer = self.peek()
        if layer is None or layer[0] != kind:
            got = layer[0] if layer is not None else "end of arch"
            raise ArchError(f"arch entry {self.i}: expected {kind!r}, got {got!r}")
        self.i += 1
        return list(layer[1:])


def decoder_plan(arch, *, int8_attention=True):
    """Validate a decoder arch and return the launch plan (a JSON-able dict).

    The decoder is ``embedding`` [+ ``positional_embedding``], then any sequence of
    pre-norm residual sub-blocks ``save_residual, <norm>, <op>, add_residual`` with
    ``<norm>`` in {rmsnorm, layernorm} and ``<op>`` one of
    ``multi_head_attention_gqa_kv`` (RoPE), ``multi_head_attention_kv``,
    ``swiglu_ffn`` or ``linear, gelu, linear``; then a final norm and the
    ``linear`` LM head. That covers every decoder the reference's decoder mode
    packs (tiny_llama_min, gqa_min, rmsnorm_swiglu_decoder, tiny_decoder_*,
    gpt2_small, tinyllama_1b, llama2_7b). Tensor references are the reference's
    staging names; int8 weights carry a companion ``<name>_scales`` tensor.
    """
    arch = [list(layer) for layer in arch]
    for layer in arch:
        if layer[0] not in DECODER_KINDS:
            raise ArchError(f"op {layer[0]!r} is not part of the decoder decode path")
    cur = _Cursor(arch)
    vocab, d, _seq = cur.take("embedding")
    plan = {
        "format": "b200-decode-plan", "version": 1,
        "vocab": vocab, "d_model": d, "token_bytes": token_bytes(vocab),
        "embedding": "Wemb0", "pos_embedding": None, "max_pos": 0,
        "eps": 1e-5, "blocks": [],
    }
    if cur.peek() and cur.peek()[0] == "positional_embedding":
        max_pos, d_pe, _ = cur.take("positional_embedding")
        if d_pe != d:
            raise ArchError("positional_embedding d_model must match the embedding")
        plan["pos_embedding"] = "Wpos0"
        plan["max_pos"] = max_pos

    cnt = {"rmsnorm": 0, "layernorm": 0, "gqa": 0, "mha": 0, "swiglu": 0, "linear": 0}

    def take_norm():
        kind = cur.peek()[0] if cur.peek() else None
        if kind == "rmsnorm":
            (nd,) = cur.take("rmsnorm")
            i = cnt["rmsnorm"]; cnt["rmsnorm"] += 1
            norm = {"kind": "rms", "g": f"Wr{i}"}
        elif kind == "layernorm":
            (nd,) = cur.take("layernorm")
            i = cnt["layernorm"]; cnt["layernorm"] += 1
            norm = {"kind": "ln", "g": f"Wn{i}", "b": f"bn{i}"}
        else:
            raise ArchError(f"arch entry {cur.i}: expected rmsnorm or layernorm, got {kind!r}")
        if nd != d:
            raise ArchError(f"norm width {nd} must equal d_model {d}")
        return norm

    max_seq = None
    while cur.peek() is not None and cur.peek()[0] == "save_residual":
        cur.take("save_residual")
        norm = take_norm()
        op = cur.peek()[0] if cur.peek() else None
        if op == "multi_head_attention_gqa_kv":
            ms, da, heads, kv_heads, theta = cur.take(op)
            tensor_specs(op, [ms, da, heads, kv_heads, theta])
            gi = cnt["gqa"]; cnt["gqa"] += 1
            blk = {"type": "attn", "kind": "gqa", "rope": True, "theta": float(theta),
                   "n_heads": heads, "n_kv_heads": kv_heads, "d_head": da // heads,
                   "dtype": "i8" if int8_attention else "f32", "bias": None}
            blk.update({p: f"Wgqa{p}{gi}" for p in "qkvo"})
            if blk["d_head"] % 2:
                raise ArchError("RoPE needs an even d_head")
        elif op == "multi_head_attention_kv":
            ms, da, heads = cur.take(op)
            tensor_specs(op, [ms, da, heads])
            mi = cnt["mha"]; cnt["mha"] += 1
            blk = {"type": "attn", "kind": "mha", "rope": False, "theta": None,
                   "n_heads": heads, "n_kv_heads": heads, "d_head": da // heads,
                   "dtype": "f32", "bias": {p: f"bm{p}{mi}" for p in "qkvo"}}
            blk.update({p: f"Wm{p}{mi}" for p in "qkvo"})
        elif op == "swiglu_ffn":
            da, ffn = cur.take(op)
            si = cnt["swiglu"]; cnt["swiglu"] += 1
            blk = {"type": "ffn", "kind": "swiglu", "d_ffn": ffn, "gate": f"Wswgate{si}",
                   "up": f"Wswup{si}", "down": f"Wswdown{si}"}
        elif op == "linear":
            da, ffn = cur.take("linear")
            li = cnt["linear"]; cnt["linear"] += 2
            cur.take("gelu")
            ffn2, out2 = cur.take("linear")
            if ffn2 != ffn or out2 != d:
                raise ArchError("linear, gelu, linear must map d_model -> d_ffn -> d_model")
            blk = {"type": "ffn", "kind": "gelu_mlp", "d_ffn": ffn, "fc1": f"W{li}",
                   "fc1_b": f"b{li}", "fc2": f"W{li + 1}", "fc2_b": f"b{li + 1}"}
        else:
            raise ArchError(f"arch entry {cur.i}: unsupported sub-block op {op!r}")
        if da != d:
            raise ArchError(f"sub-block width {da} must equal d_model {d}")
        if blk["type"] == "attn":
            if max_seq is None:
                max_seq = ms
            elif ms != max_seq:
                raise ArchError("all attention sub-blocks must share max_seq")
        blk["norm"] = norm
        cur.take("add_residual")
        plan["blocks"].append(blk)

    if max_seq is None:
        raise ArchError("decoder arch has no attention sub-block")
    plan["final_norm"] = take_norm()
    lm_in, lm_out = cur.take("linear")
    li = cnt["linear"]
    plan["lm_head"] = {"W": f"W{li}", "b": f"b{li}"}
    if cur.peek() is not None:
        raise ArchError(f"trailing arch entries after the LM head: {cur.peek()[0]!r}")
    if lm_in != d:
        raise ArchError("LM head in_features must match the embedding d_model")
    if lm_out != vocab:
        raise ArchError(f"LM head out_features ({lm_out}) must match the embedding vocab "
                        f"({vocab})")
    attn = [b for b in plan["blocks"] if b["type"] == "attn"]
    kinds = {b["kind"] for b in plan["blocks"]} | {plan["final_norm"]["kind"]}
    plan["family"] = ("llama" if kinds <= {"gqa", "swiglu", "rms"} else
                      "gpt2" if kinds <= {"mha", "gelu_mlp", "ln"} else "mixed")
    plan["max_seq"] = max_seq
    plan["n_layers"] = len(attn)
    return plan


def plan_tensor_names(plan):
    """Every tensor the runtime reads."""
    out = [plan["embedding"]]
    if plan.get("pos_embedding"):
        out.append(plan["pos_embedding"])
    for b in plan["blocks"]:
        out += [v for k, v in b["norm"].items() if k != "kind"]
        if b["type"] == "attn":
            out += [b[p] for p in "qkvo"]
            if b["bias"]:
                out += [v for v in b["bias"].values() if v]
        elif b["kind"] == "swiglu":
            out += [b["gate"], b["up"], b["down"]]
        else:
            out += [b["fc1"], b["fc1_b"], b["fc2"], b["fc2_b"]]
    out += [v for k, v in plan["final_norm"].items() if k != "kind"]
    out += [plan["lm_head"]["W"], plan["lm_head"]["b"]]
    return out
