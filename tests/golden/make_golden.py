"""Regenerate the golden fixtures under tests/golden/ from the reference itself.

Run in a container that has the reference checkout (read-only is fine; every
script runs in a temporary copy):

    python tests/golden/make_golden.py --reference /root/reference

What it writes (all small, committed):

* ``cfgT/``: the 1-block tiny Llama workload (d_model=64, 4/2 heads, head_dim 16,
  SwiGLU 172, vocab 256, max_seq 32; N(0, 0.02) weights from torch.manual_seed(0);
  8 prompt ids from torch.Generator().manual_seed(1)) as ``model.safetensors`` +
  ``arch.json`` + ``prompt.json``, and ``ref_staging/``: the reference packer's
  int8 staging files for it (``--quantize int8 --int8-attention``).
* ``<example>/`` for the reference's decoder examples tiny_llama_min, gqa_min,
  rmsnorm_swiglu_decoder, tiny_decoder_packed and tiny_decoder_2block: the files
  the example's own prepare.py writes (``synth.pt``, ``prompt.bin``,
  ``expected_tokens.bin`` = PyTorch greedy tokens), its ``arch.json``, and the
  reference packer's int8 staging files (``ref_staging/``).
* ``rope_golden.json``: the RoPE known-answer vector of
  examples/rope_min/test_rope.ari:20-25.
* ``<fixture>/ref_staging_int4/`` for cfgT, tiny_decoder_packed and
  tiny_decoder_2block: the reference packer's staging files with
  ``--int4-linear --int4-embedding`` added (``.i4`` nibble-packed codes, low
  nibble = even column, and their ``_scales.f32``). ``--int4-only`` writes just
  these, from the fixtures already committed.

Nothing under tests/ reads the reference at test time; only this script does.
"""
from __future__ import annotations

import argparse
import json
import shutil
import struct
import subprocess
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent

EXAMPLES = {
    # example -> (--int8-attention?, max_new_tokens used by its run_test*.sh)
    "tiny_llama_min": (True, 4),
    "gqa_min": (True, 4),
    "rmsnorm_swiglu_decoder": (False, 3),
    "tiny_decoder_packed": (False, 3),
    "tiny_decoder_2block": (False, 4),
}

CFG_T_ARCH = [
    ["embedding", 256, 64, 1],
    ["save_residual"], ["rmsnorm", 64],
    ["multi_head_attention_gqa_kv", 32, 64, 4, 2, 10000.0],
    ["add_residual"],
    ["save_residual"], ["rmsnorm", 64], ["swiglu_ffn", 64, 172], ["add_residual"],
    ["rmsnorm", 64],
    ["linear", 64, 256],
]


def cfg_t_state_dict():
    """N(0, 0.02) weights in arch order from torch.manual_seed(0); norm gains 1;
    LM-head bias 0 (the reference's prepare scripts synthesise a zero bias for the
    head, e.g. examples/tinyllama_1b/prepare.py:155-158)."""
    import torch
    torch.manual_seed(0)
    d, kv, ffn, vocab = 64, 32, 172, 256
    g = lambda *s: (torch.randn(*s) * 0.02).float()
    sd = {"embed.weight": g(vocab, d)}
    p = "model.layers.0"
    sd[f"{p}.input_layernorm.weight"] = torch.ones(d)
    sd[f"{p}.self_attn.q_proj.weight"] = g(d, d)
    sd[f"{p}.self_attn.k_proj.weight"] = g(kv, d)
    sd[f"{p}.self_attn.v_proj.weight"] = g(kv, d)
    sd[f"{p}.self_attn.o_proj.weight"] = g(d, d)
    sd[f"{p}.post_attention_layernorm.weight"] = torch.ones(d)
    sd[f"{p}.mlp.gate_proj.weight"] = g(ffn, d)
    sd[f"{p}.mlp.up_proj.weight"] = g(ffn, d)
    sd[f"{p}.mlp.down_proj.weight"] = g(d, ffn)
    sd["model.norm.weight"] = torch.ones(d)
    sd["fc1.weight"] = g(vocab, d)
    sd["fc1.bias"] = torch.zeros(vocab)
    prompt = torch.randint(0, vocab, (8,), generator=torch.Generator().manual_seed(1)).tolist()
    return sd, prompt


def run_ref_packer(ref, workdir, checkpoint, arch_path, prompt_bin, int8_attention, max_new, out, extra=()):
    cmd = [sys.executable, str(ref / "tools" / "aricode_pack.py"), "--checkpoint", str(checkpoint),
           "--arch", str(arch_path), "--keys", "fc{idx_plus_1}.{kind}",
           "--input-format", "embedded", "--input-file", str(prompt_bin), "--embed",
           "--no-argmax", "--quantize", "int8", "--max-new-tokens", str(max_new),
           "--out", str(workdir / out)]
    if int8_attention:
        cmd.append("--int8-attention")
    cmd += list(extra)
    subprocess.run(cmd, check=True, cwd=workdir, stdout=subprocess.DEVNULL)
    return cmd


def collect_staging(workdir, out, dest):
    dest.mkdir(parents=True, exist_ok=True)
    for f in sorted(workdir.glob(f"{out}_*")):
        if f.suffix in (".i8", ".i4", ".f32"):
            shutil.copy(f, dest / f.name[len(out) + 1:])


INT4_FIXTURES = {"cfgT": ("model.safetensors", True), "tiny_decoder_packed": ("synth.pt", False),
                 "tiny_decoder_2block": ("synth.pt", False)}


def int4_staging(ref, td):
    """ref_staging_int4/ of the committed fixtures (the reference packer with
    --int4-linear --int4-embedding)."""
    for name, (ckpt, i8attn) in INT4_FIXTURES.items():
        src = HERE / name
        work = td / f"{name}_int4"
        work.mkdir()
        prompt = json.loads((src / "prompt.json").read_text())["prompt"] if name == "cfgT" else \
            list((src / "prompt.bin").read_bytes())
        (work / "prompt.bin").write_bytes(bytes(prompt))
        run_ref_packer(ref, work, src / ckpt, src / "arch.json", work / "prompt.bin", i8attn, 4, name,
                       extra=("--int4-linear", "--int4-embedding"))
        dest = src / "ref_staging_int4"
        if dest.exists():
            shutil.rmtree(dest)
        collect_staging(work, name, dest)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    ap.add_argument("--int4-only", action="store_true")
    a = ap.parse_args()
    ref = Path(a.reference)
    if a.int4_only:
        with tempfile.TemporaryDirectory() as td:
            int4_staging(ref, Path(td))
        return
    manifest = {"generated_by": "tests/golden/make_golden.py", "fixtures": {}}

    with tempfile.TemporaryDirectory() as td:
        td = Path(td)
        # ---------------- cfgT
        from safetensors.torch import save_file
        sd, prompt = cfg_t_state_dict()
        dest = HERE / "cfgT"
        dest.mkdir(exist_ok=True)
        save_file(sd, str(dest / "model.safetensors"))
        (dest / "arch.json").write_text(json.dumps(CFG_T_ARCH, indent=1))
        (dest / "prompt.json").write_text(json.dumps({"prompt": prompt, "max_new": 16}))
        work = td / "cfgT"
        work.mkdir()
        (work / "prompt.bin").write_bytes(bytes(prompt))
        cmd = run_ref_packer(ref, work, dest / "model.safetensors", dest / "arch.json",
                             work / "prompt.bin", True, 16, "cfgT")
        if (dest / "ref_staging").exists():
            shutil.rmtree(dest / "ref_staging")
        collect_staging(work, "cfgT", dest / "ref_staging")
        # the flags as run, with this checkout's and the scratch folder's paths
        # written relative to the repository / as <work>
        root = str(HERE.parents[1]) + "/"
        manifest["fixtures"]["cfgT"] = {"pack_flags": [a.replace(str(td), "<work>").replace(root, "")
                                                       for a in map(str, cmd[3:])]}

        # ---------------- reference decoder examples
        for ex, (i8attn, max_new) in EXAMPLES.items():
            work = td / ex
            shutil.copytree(ref / "examples" / ex, work)
            subprocess.run([sys.executable, "prepare.py"], check=True, cwd=work,
                           stdout=subprocess.DEVNULL)
            run_ref_packer(ref, work, work / "synth.pt", work / "arch.json",
                           work / "prompt.bin", i8attn, max_new, ex)
            dest = HERE / ex
            if dest.exists():
                shutil.rmtree(dest)
            dest.mkdir()
            for f in ("synth.pt", "prompt.bin", "expected_tokens.bin", "arch.json"):
                shutil.copy(work / f, dest / f)
            collect_staging(work, ex, dest / "ref_staging")
            exp = list(struct.unpack(f"<{(work / 'expected_tokens.bin').stat().st_size // 4}i",
                                     (work / "expected_tokens.bin").read_bytes()))
            manifest["fixtures"][ex] = {"int8_attention": i8attn, "max_new": max_new,
                                        "expected_tokens": exp,
                                        "source": f"examples/{ex}/prepare.py"}
        int4_staging(ref, td)

    (HERE / "rope_golden.json").write_text(json.dumps({
        "source": "examples/rope_min/test_rope.ari:20-25,42",
        "max_seq": 4, "d_head": 4, "theta": 10000.0, "pos": 1,
        "input": [1.0, 2.0, 3.0, 4.0],
        "expected": [-1.1426396637476532, 1.9220755965441760, 2.9598506679133294,
                     4.0297995016691610],
        "tol": 1e-5}, indent=1))
    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1))
    print(json.dumps(manifest, indent=1))


if __name__ == "__main__":
    main()
