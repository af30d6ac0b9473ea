"""Synthetic workloads: the decoder configs the decode path is measured on, as
reference arch JSON, plus the tensor specs a synthetic model is generated from.

Weights of a synthetic model come from a counter-based generator (splitmix64 of
(seed, tensor id, element index) -> centred sum of four 16-bit uniforms, scaled
to std 0.02), quantised per row exactly like the packer. The same generator runs
on the GPU (b2_create_synthetic) and on the host in the oracle, so both see
bit-identical weights without staging a multi-GB checkpoint. Tensor id =
FNV-1a-64 of the tensor's staging name. Norm gains are 1, LayerNorm shifts and
the LM-head bias 0, other biases and positional rows random.

Stand-in for public checkpoints: the configs below use random weights of the
named architecture (no checkpoint download is possible or needed).
"""
from __future__ import annotations

from . import arch as A


def llama_arch(vocab, d, n_layers, heads, kv_heads, ffn, max_seq, theta=10000.0):
    a = [["embedding", vocab, d, 1]]
    for _ in range(n_layers):
        a += [["save_residual"], ["rmsnorm", d],
              ["multi_head_attention_gqa_kv", max_seq, d, heads, kv_heads, theta],
              ["add_residual"],
              ["save_residual"], ["rmsnorm", d], ["swiglu_ffn", d, ffn], ["add_residual"]]
    a += [["rmsnorm", d], ["linear", d, vocab]]
    return a


def gpt2_arch(vocab, d, n_layers, heads, ffn, max_seq, max_pos=1024):
    a = [["embedding", vocab, d, 1], ["positional_embedding", max_pos, d, 1]]
    for _ in range(n_layers):
        a += [["save_residual"], ["layernorm", d], ["multi_head_attention_kv", max_seq, d, heads],
              ["add_residual"],
              ["save_residual"], ["layernorm", d], ["linear", d, ffn], ["gelu"], ["linear", ffn, d],
              ["add_residual"]]
    a += [["layernorm", d], ["linear", d, vocab]]
    return a


# name -> (arch builder kwargs, prompt_len, new_tokens, batch)
CONFIGS = {
    # 1-block tiny Llama: d=64, 4 heads / 2 kv heads, head_dim 16, SwiGLU 172, vocab 256
    "tiny-llama": dict(kind="llama", vocab=256, d=64, n_layers=1, heads=4, kv_heads=2, ffn=172,
                       max_seq=32, prompt=8, new=16, batch=1),
    # GPT-2-small: 12 x (768, 12 heads, GELU 3072), learned positions, vocab 50257
    "gpt2-small": dict(kind="gpt2", vocab=50257, d=768, n_layers=12, heads=12, ffn=3072,
                       max_seq=128, prompt=8, new=16, batch=1),
    # TinyLlama-1.1B: 22 x (2048, 32 heads / 4 kv heads, SwiGLU 5632), vocab 32000
    "tinyllama-1.1b": dict(kind="llama", vocab=32000, d=2048, n_layers=22, heads=32, kv_heads=4,
                           ffn=5632, max_seq=2048, prompt=128, new=128, batch=1),
    # Llama-2-7B: 32 x (4096, 32 heads MHA, SwiGLU 11008), vocab 32000; 512 + 256 tokens
    "llama2-7b": dict(kind="llama", vocab=32000, d=4096, n_layers=32, heads=32, kv_heads=32,
                      ffn=11008, max_seq=768, prompt=512, new=256, batch=1),
    # Llama-2-7B batched decode: 64 sequences x (1024 + 128)
    "llama2-7b-b64": dict(kind="llama", vocab=32000, d=4096, n_layers=32, heads=32, kv_heads=32,
                          ffn=11008, max_seq=1152, prompt=1024, new=128, batch=64),
}


def config_arch(name, n_layers=None, max_seq=None):
    c = dict(CONFIGS[name])
    if n_layers is not None:
        c["n_layers"] = n_layers
    if max_seq is not None:
        c["max_seq"] = max_seq
    if c["kind"] == "llama":
        return llama_arch(c["vocab"], c["d"], c["n_layers"], c["heads"], c["kv_heads"], c["ffn"],
                          c["max_seq"])
    return gpt2_arch(c["vocab"], c["d"], c["n_layers"], c["heads"], c["ffn"], c["max_seq"])


def config_plan(name, n_layers=None, max_seq=None):
    c = CONFIGS[name]
    return A.decoder_plan(config_arch(name, n_layers, max_seq),
                          int8_attention=(c["kind"] == "llama"))


def tensor_specs(plan):
    """[(name, dtype 'i8'|'f32', shape tuple, init 'rand'|'ones'|'zeros')] in plan order;
    the C++ runtime's plan_needs() enumerates the same list."""
    d, vocab = plan["d_model"], plan["vocab"]
    out = []

    def norm(n):
        out.append((n["g"], "f32", (d,), "ones"))
        if n["kind"] == "ln":
            out.append((n["b"], "f32", (d,), "zeros"))

    out.append((plan["embedding"], "i8", (vocab, d), "rand"))
    if plan.get("pos_embedding"):
        out.append((plan["pos_embedding"], "f32", (plan["max_pos"], d), "rand"))
    for b in plan["blocks"]:
        norm(b["norm"])
        if b["type"] == "attn":
            qd, kd = b["n_heads"] * b["d_head"], b["n_kv_heads"] * b["d_head"]
            dt = b["dtype"]
            out += [(b["q"], dt, (qd, d), "rand"), (b["k"], dt, (kd, d), "rand"),
                    (b["v"], dt, (kd, d), "rand"), (b["o"], dt, (d, qd), "rand")]
            if b.get("bias"):
                bs = b["bias"]
                out += [(bs[p], "f32", (n,), "rand") for p, n in (("q", qd), ("k", kd), ("v", kd), ("o", d))
                        if bs.get(p)]
        elif b["kind"] == "swiglu":
            f = b["d_ffn"]
            out += [(b["gate"], "i8", (f, d), "rand"), (b["up"], "i8", (f, d), "rand"),
                    (b["down"], "i8", (d, f), "rand")]
        else:
            f = b["d_ffn"]
            out += [(b["fc1"], "i8", (f, d), "rand"), (b["fc1_b"], "f32", (f,), "rand"),
                    (b["fc2"], "i8", (d, f), "rand"), (b["fc2_b"], "f32", (d,), "rand")]
    norm(plan["final_norm"])
    out.append((plan["lm_head"]["W"], "i8", (vocab, d), "rand"))
    out.append((plan["lm_head"]["b"], "f32", (vocab,), "zeros"))
    return out


def weight_bytes(plan):
    """Algorithmic weight bytes streamed per decoded token: every int8 matrix
    (codes + f32 row scales), f32 matrices, biases and norm parameters once, plus
    one embedding row (codes + scale) and one positional row."""
    tot = 0
    d = plan["d_model"]
    for name, dt, shape, _ in tensor_specs(plan):
        if name == plan["embedding"]:
            tot += d + 4
        elif name == plan.get("pos_embedding"):
            tot += 4 * d
        elif dt == "i8":
            tot += shape[0] * shape[1] + 4 * shape[0]
        else:
            n = 1
            for s in shape:
                n *= s
            tot += 4 * n
    return tot


def kv_bytes(plan, pos):
    """KV bytes for the token at position pos: read rows 0..pos, write row pos."""
    per = sum(2 * b["n_kv_heads"] * b["d_head"] * 4 for b in plan["blocks"] if b["type"] == "attn")
    return per * (pos + 1) + per


def bytes_per_token(plan, pos):
    return weight_bytes(plan) + kv_bytes(plan, pos)
