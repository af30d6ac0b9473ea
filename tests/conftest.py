"""Shared fixtures. GPU tests are marked ``gpu``; everything else runs on CPU."""
import importlib
import json
import os
import struct
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = ROOT / "tests" / "golden"
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def pkg():
    return importlib.import_module("aricode-ml_b200")


@pytest.fixture(scope="session")
def oracle():
    import oracle as O
    O.build()
    return O


def load_example(pkg, name):
    """(plan, tensors, prompt, max_new, expected_tokens) for a golden fixture dir."""
    man = json.loads((GOLDEN / "manifest.json").read_text())
    d = GOLDEN / name
    arch = json.loads((d / "arch.json").read_text())
    if name == "cfgT":
        sd = pkg.pack.load_state_dict(d / "model.safetensors")
        pr = json.loads((d / "prompt.json").read_text())
        plan, tensors = pkg.pack.pack(arch, sd, int8_attention=True)
        return plan, tensors, pr["prompt"], pr["max_new"], None
    info = man["fixtures"][name]
    sd = pkg.pack.load_state_dict(d / "synth.pt")
    plan, tensors = pkg.pack.pack(arch, sd, int8_attention=info["int8_attention"])
    prompt = list((d / "prompt.bin").read_bytes())
    return plan, tensors, prompt, info["max_new"], info["expected_tokens"]


EXAMPLES = ["tiny_llama_min", "gqa_min", "rmsnorm_swiglu_decoder", "tiny_decoder_packed",
            "tiny_decoder_2block"]


@pytest.fixture
def tmp_out(tmp_path):
    return tmp_path
