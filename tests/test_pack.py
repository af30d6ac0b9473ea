"""Packer parity with the reference packer, plan and blob format (no GPU)."""
import json

import numpy as np
import pytest

from conftest import EXAMPLES, GOLDEN, load_example


def _staging_diffs(tensors, d):
    bad = []
    for f in sorted((d / "ref_staging").iterdir()):
        t = tensors.get(f.stem)
        if t is None:
            bad.append(("missing", f.stem))
        elif np.ascontiguousarray(t).tobytes() != f.read_bytes():
            bad.append(("differs", f.stem))
    return bad


@pytest.mark.parametrize("name", ["cfgT"] + EXAMPLES)
def test_codes_scales_bytes_equal_reference_packer(pkg, name):
    """Every staging file the reference packer wrote (int8 codes, f32 scales,
    biases, norms) is byte-identical to ours (aricode_pack.py:3252-3416)."""
    plan, tensors, *_ = load_example(pkg, name)
    assert _staging_diffs(tensors, GOLDEN / name) == []


def test_quantiser_edge_rows(pkg):
    W = np.array([[0, 0, 0], [1.0, -2.0, 0.5], [2.5 * 127 / 127, -1e-30, 0]], np.float32)
    q, s = pkg.pack.quantize_rows(W)
    assert s[0] == 0 and (q[0] == 0).all()                 # all-zero row keeps scale 0
    assert q[1].tolist() == [64, -127, 32]                  # round half to even: 63.5 -> 64
    assert q.dtype == np.int8 and s.dtype == np.float32


def test_blob_roundtrip_and_checksum(pkg, tmp_path):
    plan, tensors, *_ = load_example(pkg, "tiny_decoder_2block")
    path = tmp_path / "m.b2blob"
    pkg.blob.write_blob(path, tensors, plan)
    plan2, t2 = pkg.blob.read_blob(path)
    assert plan2 == json.loads(json.dumps(plan))
    for k, v in tensors.items():
        assert np.array_equal(np.asarray(t2[k]), v), k
    raw = bytearray(path.read_bytes())
    raw[-1] ^= 0xFF
    path.write_bytes(bytes(raw))
    with pytest.raises(ValueError, match="checksum"):
        pkg.blob.read_blob(path)


def test_blob_rows_are_16_byte_aligned(pkg, tmp_path):
    plan, tensors, *_ = load_example(pkg, "cfgT")        # swiglu down: 64 x 172
    ents = pkg.blob.write_blob(tmp_path / "m.b2blob", tensors, plan)
    for e in ents:
        assert e.offset % 256 == 0
        if len(e.shape) == 2 and e.dtype == pkg.blob.DT_I8:
            assert e.ld % 16 == 0


def test_cli_writes_blob_and_plan(pkg, tmp_path):
    d = GOLDEN / "cfgT"
    rc = pkg.pack.main(["--checkpoint", str(d / "model.safetensors"), "--arch", str(d / "arch.json"),
                        "--quantize", "int8", "--int8-attention", "--out", str(tmp_path / "m")])
    assert rc == 0
    plan = json.loads((tmp_path / "m.plan.json").read_text())
    assert plan["family"] == "llama" and plan["vocab"] == 256 and plan["max_seq"] == 32
    assert (tmp_path / "m.b2blob").exists()


def _cli(pkg, tmp_path, *extra):
    d = GOLDEN / "cfgT"
    return pkg.pack.main(["--checkpoint", str(d / "model.safetensors"), "--arch", str(d / "arch.json"),
                          "--quantize", "int8", "--int8-attention", "--out", str(tmp_path / "m"),
                          *extra])


def test_cli_sampling_flags_reach_the_plan(pkg, tmp_path):
    assert _cli(pkg, tmp_path, "--sample", "topk:40:0.8", "--rng-seed", "77", "--eos-token", "2",
                "--max-prompt-tokens", "20") == 0
    g = json.loads((tmp_path / "m.plan.json").read_text())["generation"]
    assert (g["sample_mode"], g["top_k"], g["temperature"], g["rng_seed"]) == (2, 40, 0.8, 77)
    assert g["eos_token"] == 2 and g["max_prompt_tokens"] == 20


@pytest.mark.parametrize("extra", [["--sample", "nucleus:0.9"], ["--sample", "topk:5"], ["--profile"],
                                   ["--no-argmax"], ["--n-test", "5"], ["--input-format", "mnist"],
                                   ["--input-format", "embedded"], ["--max-prompt-tokens", "0"],
                                   ["--target", "aric"], ["--infer-arch"]])
def test_cli_flags_that_cannot_work_are_refused(pkg, tmp_path, extra):
    with pytest.raises(pkg.pack.PackError):
        _cli(pkg, tmp_path, *extra)


def test_missing_key_is_a_pack_error(pkg):
    arch = json.loads((GOLDEN / "cfgT" / "arch.json").read_text())
    sd = pkg.pack.load_state_dict(GOLDEN / "cfgT" / "model.safetensors")
    sd = {k: v for k, v in sd.items() if "o_proj" not in k}
    with pytest.raises(SystemExit, match="o_proj"):
        pkg.pack.pack(arch, sd, int8_attention=True)


def test_shape_mismatch_is_a_pack_error(pkg):
    arch = json.loads((GOLDEN / "cfgT" / "arch.json").read_text())
    arch[-1] = ["linear", 64, 255]
    sd = pkg.pack.load_state_dict(GOLDEN / "cfgT" / "model.safetensors")
    with pytest.raises((SystemExit, ValueError)):
        pkg.pack.pack(arch, sd, int8_attention=True)


def test_decoder_plan_rejects_non_decoder_ops(pkg):
    with pytest.raises(pkg.arch.ArchError):
        pkg.arch.decoder_plan([["linear", 784, 10]])
    with pytest.raises(pkg.arch.ArchError):
        pkg.arch.decoder_plan([["embedding", 8, 4, 1], ["conv2d_3x3_p1", 1, 2]])


def test_keys_template_and_hf_fallbacks(pkg):
    """--keys template ({idx}, {idx_plus_1}, {kind}) and the plain gqa/swiglu test-rig keys."""
    import torch
    torch.manual_seed(0)
    arch = pkg.synth.config_arch("tiny-llama")
    sd = {"embed.weight": torch.randn(256, 64), "gqa0.q.weight": torch.randn(64, 64),
          "gqa0.k.weight": torch.randn(32, 64), "gqa0.v.weight": torch.randn(32, 64),
          "gqa0.o.weight": torch.randn(64, 64), "rmsnorm0.weight": torch.ones(64),
          "rmsnorm1.weight": torch.ones(64), "rmsnorm2.weight": torch.ones(64),
          "swiglu0.gate.weight": torch.randn(172, 64), "swiglu0.up.weight": torch.randn(172, 64),
          "swiglu0.down.weight": torch.randn(64, 172),
          "head.0.weight": torch.randn(256, 64), "head.0.bias": torch.zeros(256)}
    plan, tensors = pkg.pack.pack(arch, sd, keys="head.{idx}.{kind}", int8_attention=True)
    assert "W0" in tensors and tensors["Wgqaq0"].dtype == np.int8


@pytest.mark.parametrize("name,gb", [("llama2-7b", 6.614), ("tinyllama-1.1b", 1.036)])
def test_algorithmic_weight_bytes(pkg, name, gb):
    plan = pkg.synth.config_plan(name)
    assert abs(pkg.synth.weight_bytes(plan) / 1e9 - gb) < 0.01


def test_gqa_biases_are_staged_when_the_checkpoint_has_them(pkg):
    import torch
    d = GOLDEN / "tiny_llama_min"
    arch = json.loads((d / "arch.json").read_text())
    sd = dict(pkg.pack.load_state_dict(d / "synth.pt"))
    sd["model.layers.0.self_attn.k_proj.bias"] = torch.ones(8)
    plan, tensors = pkg.pack.pack(arch, sd)
    b = [blk for blk in plan["blocks"] if blk.get("kind") == "gqa"][0]["bias"]
    assert b == {"q": None, "k": "bgqak0", "v": None, "o": None}
    assert np.array_equal(tensors["bgqak0"], np.ones(8, np.float32))
    sd["model.layers.0.self_attn.k_proj.bias"] = torch.ones(7)
    with pytest.raises(pkg.pack.PackError):
        pkg.pack.pack(arch, sd)


@pytest.mark.parametrize("name", ["cfgT", "tiny_decoder_packed", "tiny_decoder_2block"])
def test_int4_codes_and_scales_bytes_equal_reference_packer(pkg, name):
    """--int4-linear --int4-embedding: every staging file the reference packer wrote
    (.i4 nibble-packed codes, their scales, and the int8/f32 rest) is byte-identical
    (aricode_pack.py:3299-3355)."""
    d = GOLDEN / name
    arch = json.loads((d / "arch.json").read_text())
    ckpt = "model.safetensors" if name == "cfgT" else "synth.pt"
    sd = pkg.pack.load_state_dict(d / ckpt)
    plan, tensors = pkg.pack.pack(arch, sd, int8_attention=(name == "cfgT"), int4_linear=True,
                                  int4_embedding=True)
    bad = []
    for f in sorted((d / "ref_staging_int4").iterdir()):
        t = tensors.get(f.stem)
        if t is None or np.ascontiguousarray(t).tobytes() != f.read_bytes():
            bad.append(f.name)
    assert bad == []
    assert tensors[plan["embedding"]].dtype == np.uint8


def test_int4_blob_roundtrip_and_oracle_matvec(pkg, oracle, tmp_path):
    d = GOLDEN / "cfgT"
    arch = json.loads((d / "arch.json").read_text())
    sd = pkg.pack.load_state_dict(d / "model.safetensors")
    plan, tensors = pkg.pack.pack(arch, sd, int8_attention=True, int4_linear=True, int4_embedding=True)
    pkg.blob.write_blob(tmp_path / "m.b2blob", tensors, plan)
    plan2, t2 = pkg.blob.read_blob(tmp_path / "m.b2blob")
    W = plan["lm_head"]["W"]
    assert t2[W].dtype == np.uint8 and np.array_equal(t2[W], tensors[W])
    # the int4 matvec is the int8 matvec of the unpacked codes
    n = plan["d_model"]
    x = np.random.default_rng(0).standard_normal(n).astype(np.float32)
    codes = np.stack([oracle.unpack_i4(r, n) for r in tensors[W]])
    assert codes.min() >= -8 and codes.max() <= 7
    assert np.array_equal(oracle.gemv_i4(tensors[W], tensors[W + "_scales"], x, n),
                          oracle.gemv_i8(codes, tensors[W + "_scales"], x))
    # and the decoder runs on it
    om = oracle.OracleModel(plan2, t2)
    assert len(om.generate([1, 2, 3], 5)) == 5


def test_int4_odd_rows_are_refused(pkg):
    with pytest.raises(pkg.pack.PackError):
        pkg.pack.build_tensors([["linear", 3, 2]], [("linear", 0, "", np.ones((2, 3), np.float32), None)],
                               int4_linear=True)
