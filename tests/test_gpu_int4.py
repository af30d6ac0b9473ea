"""int4 per-row weights (--int4-linear / --int4-embedding, the reference's nibble
format): the GPU int4 GEMV streams packed rows and must equal the oracle's
restatement (the int8 dot over the unpacked codes) bit for bit, and packed models
must decode with the oracle's ids and logits."""
import json

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,n", [(256, 64), (5, 16), (768, 3072), (3072, 768), (32000, 4096), (1000, 8192)])
def test_int4_gemv_matches_oracle(pkg, oracle, m, n):
    import torch
    rng = np.random.default_rng(m + n)
    W = (rng.standard_normal((m, n)) * 0.02).astype(np.float32)
    q, s = pkg.pack.quantize_rows_i4(W)
    ld = (q.shape[1] + 15) // 16 * 16
    qp = np.zeros((m, ld), np.uint8)
    qp[:, :q.shape[1]] = q
    x = rng.standard_normal(n).astype(np.float32)
    b = rng.standard_normal(m).astype(np.float32)
    y = pkg.runtime.gemv_i4(torch.from_numpy(qp).cuda(), torch.from_numpy(s).cuda(), torch.from_numpy(x).cuda(), n,
                            bias=torch.from_numpy(b).cuda()).cpu().numpy()
    ref = oracle.gemv_i4(q, s, x, n)
    assert np.array_equal(y, (ref + b).astype(np.float32))


@pytest.mark.parametrize("name,lin,emb", [("cfgT", True, True), ("cfgT", False, True), ("tiny_decoder_packed", True, True),
                                          ("tiny_decoder_2block", True, False)])
def test_int4_packed_models_match_oracle(pkg, oracle, name, lin, emb, tmp_path):
    d = GOLDEN / name
    arch = json.loads((d / "arch.json").read_text())
    sd = pkg.pack.load_state_dict(d / ("model.safetensors" if name == "cfgT" else "synth.pt"))
    plan, tensors = pkg.pack.pack(arch, sd, int8_attention=(name == "cfgT"), int4_linear=lin, int4_embedding=emb)
    pkg.blob.write_blob(tmp_path / "m.b2blob", tensors, plan)
    prompt = [1, 5, 2, 7] if name != "cfgT" else [3, 14, 15, 92, 65]
    new = min(8, plan["max_seq"] - len(prompt))
    om = oracle.OracleModel(plan, tensors)
    ref = om.generate(prompt, new)
    dec = pkg.runtime.Decoder(tmp_path / "m.b2blob")
    assert dec.generate(prompt, new) == ref
    om.reset()
    dec.reset()
    for t in prompt + ref[:-1]:
        r_tok, r_log = om.step(t)
        g_tok, g_log = dec.step(t, want_logits=True)
        assert g_tok == r_tok and np.array_equal(g_log, r_log)
    dec.close()
