"""The stdin-tokens front end (aricode-ml_b200/b2run, started like the reference's
packed binary by tools/run_decoder.py): wire-format checks that stop before any GPU
work run on the CPU; decoding through it runs on the GPU."""
import struct
import subprocess

import numpy as np
import pytest

from conftest import GOLDEN


def pack_tokens(tokens, tb, seed):
    """The reference wrapper's payload (run_decoder.py:50-59): [u32 len][u32 seed][ids]."""
    fmt = {1: "B", 2: "<H", 4: "<I"}[tb]
    return struct.pack("<II", len(tokens), seed) + b"".join(struct.pack(fmt, t) for t in tokens)


def run(launcher, payload, timeout=300):
    r = subprocess.run(["./" + launcher.name], cwd=launcher.parent, input=payload, capture_output=True,
                       timeout=timeout)
    return r.returncode, [int(x) for x in r.stdout.decode().split()], r.stderr.decode()


@pytest.fixture
def packed(pkg, tmp_path):
    def make(*extra):
        d = GOLDEN / "cfgT"
        out = tmp_path / "tiny_chat"
        assert pkg.pack.main(["--checkpoint", str(d / "model.safetensors"), "--arch", str(d / "arch.json"),
                              "--quantize", "int8", "--int8-attention", "--max-new-tokens", "10",
                              "--out", str(out), *extra]) == 0
        assert out.is_symlink()
        return out
    return make


@pytest.mark.parametrize("payload,what", [
    (b"\x03\x00", "header"),
    (struct.pack("<II", 4, 0) + b"\x01\x02", "inside the prompt"),
    (struct.pack("<II", 600, 0) + bytes(600), "max-prompt-tokens"),
])
def test_wire_format_errors(packed, payload, what):
    rc, ids, err = run(packed(), payload)
    assert rc == 2 and ids == [] and what in err


def test_prompt_cap_from_the_packer(packed):
    out = packed("--max-prompt-tokens", "4")
    rc, _, err = run(out, pack_tokens([1, 2, 3, 4, 5], 1, 0))
    assert rc == 2 and "max-prompt-tokens" in err


@pytest.mark.gpu
@pytest.mark.parametrize("sample", ["greedy", "topk:20:0.9"])
def test_front_end_decodes_like_the_oracle(pkg, oracle, packed, sample):
    out = packed("--sample", sample, "--eos-token", "-1" if sample == "greedy" else "7")
    plan, tensors = pkg.blob.read_blob(out.with_suffix(".b2blob"))
    om = oracle.OracleModel(plan, tensors)
    prompt = [3, 14, 15, 92, 65]
    eos = -1 if sample == "greedy" else 7
    for seed in (1, 4242):
        om.reset()
        ref = om.generate_sampled(prompt, 10, sample, seed=seed, eos=eos)
        rc, ids, err = run(out, pack_tokens(prompt, 1, seed))
        assert rc == 0, err
        assert ids == ref
