"""Kernel-level parity: every CUDA kernel bit-identical to the CPU oracle.

Calls go through the C ABI (libb2dec.so) with torch tensors used only as device
memory. The bar is exact equality of the f32 results (same operation order on
both sides), not a tolerance.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch


def _dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _pad16(q):
    m, n = q.shape
    ld = (n + 15) // 16 * 16
    out = np.zeros((m, ld), np.int8)
    out[:, :n] = q
    return out


@pytest.mark.parametrize("m,n", [(1, 16), (7, 172), (64, 64), (300, 768), (1000, 2048),
                                 (4096, 4096), (4096, 11008), (11008, 4096), (50257, 768)])
def test_gemv_i8_bit_exact(torch_cuda, pkg, oracle, m, n):
    torch = torch_cuda
    rng = np.random.default_rng(m * 7 + n)
    q = rng.integers(-128, 128, (m, n), dtype=np.int8)
    s = (rng.random(m, dtype=np.float32) * 1e-3).astype(np.float32)
    x = rng.standard_normal(n).astype(np.float32)
    ref = oracle.gemv_i8(q, s, x)
    y = pkg.runtime.gemv_i8(_dev(torch, _pad16(q)), _dev(torch, s), _dev(torch, x), n=n)
    torch.cuda.synchronize()
    assert np.array_equal(y.cpu().numpy(), ref)


def test_gemv_i8_bias(torch_cuda, pkg, oracle):
    torch = torch_cuda
    rng = np.random.default_rng(3)
    q = rng.integers(-128, 128, (333, 512), dtype=np.int8)
    s = rng.random(333, dtype=np.float32)
    x = rng.standard_normal(512).astype(np.float32)
    b = rng.standard_normal(333).astype(np.float32)
    y = pkg.runtime.gemv_i8(_dev(torch, q), _dev(torch, s), _dev(torch, x), bias=_dev(torch, b))
    assert np.array_equal(y.cpu().numpy(), oracle.gemv_i8(q, s, x) + b)


@pytest.mark.parametrize("m,n", [(8, 8), (768, 768), (2304, 768), (100, 1000)])
def test_gemv_f32_bit_exact(torch_cuda, pkg, oracle, m, n):
    torch = torch_cuda
    rng = np.random.default_rng(n)
    W = (rng.standard_normal((m, n)) * 0.02).astype(np.float32)
    x = rng.standard_normal(n).astype(np.float32)
    ld = (n + 3) // 4 * 4
    Wp = np.zeros((m, ld), np.float32); Wp[:, :n] = W
    y = pkg.runtime.gemv_f32(_dev(torch, Wp), _dev(torch, x), n=n)
    assert np.array_equal(y.cpu().numpy(), oracle.gemv_f32(W, x) + np.float32(0.0))


@pytest.mark.parametrize("d", [8, 64, 768, 4096, 5000])
def test_norms_bit_exact(torch_cuda, pkg, oracle, d):
    torch = torch_cuda
    rng = np.random.default_rng(d)
    x = (rng.standard_normal(d) * 3).astype(np.float32)
    g = rng.standard_normal(d).astype(np.float32)
    b = rng.standard_normal(d).astype(np.float32)
    assert np.array_equal(pkg.runtime.rmsnorm(_dev(torch, x), _dev(torch, g)).cpu().numpy(),
                          oracle.rmsnorm(x, g))
    assert np.array_equal(pkg.runtime.layernorm(_dev(torch, x), _dev(torch, g), _dev(torch, b)).cpu().numpy(),
                          oracle.layernorm(x, g, b))


def test_rope_bit_exact_and_golden(torch_cuda, pkg, oracle):
    torch = torch_cuda
    tab = oracle.rope_table(64, 128, 10000.0)
    rng = np.random.default_rng(1)
    v = rng.standard_normal(4 * 128).astype(np.float32)
    dv = _dev(torch, v)
    pkg.runtime.rope_apply(dv, _dev(torch, tab), 37, 128)
    ref = np.concatenate([oracle.rope_apply(v[i * 128:(i + 1) * 128], tab, 37) for i in range(4)])
    assert np.array_equal(dv.cpu().numpy(), ref)
    t4 = oracle.rope_table(4, 4, 10000.0)
    g = _dev(torch, np.array([1, 2, 3, 4], np.float32))
    pkg.runtime.rope_apply(g, _dev(torch, t4), 1, 4)
    exp = np.array([-1.1426396637476532, 1.9220755965441760, 2.9598506679133294, 4.0297995016691610])
    assert np.max(np.abs(g.cpu().numpy() - exp)) < 1e-5


@pytest.mark.parametrize("H,KVH,dh,n,max_seq", [
    (1, 1, 8, 4, 4), (1, 1, 8, 1, 9), (4, 2, 16, 7, 32), (4, 2, 16, 32, 32),
    (12, 12, 64, 128, 128), (12, 12, 64, 65, 128), (32, 4, 64, 200, 2048),
    (32, 32, 128, 640, 768), (32, 32, 128, 768, 768)])
def test_attention_bit_exact(torch_cuda, pkg, oracle, H, KVH, dh, n, max_seq):
    torch = torch_cuda
    rng = np.random.default_rng(H * 1000 + n)
    q = (rng.standard_normal(H * dh) * 0.3).astype(np.float32)
    K = rng.standard_normal((KVH, max_seq, dh)).astype(np.float32)
    V = rng.standard_normal((KVH, max_seq, dh)).astype(np.float32)
    ref = oracle.attn_decode(q, K, V, H, KVH, dh, n, max_seq)
    ws = torch.zeros(pkg.runtime.attn_workspace_bytes(H, KVH, dh, max_seq), dtype=torch.uint8,
                     device="cuda")
    for _ in range(2):           # the workspace is left reusable (counters back at zero)
        out = pkg.runtime.attn_decode(_dev(torch, q), _dev(torch, K), _dev(torch, V), H, KVH, dh, n,
                                      max_seq, workspace=ws)
        assert np.array_equal(out.cpu().numpy(), ref)


@pytest.mark.parametrize("vals,exp", [
    ([0.1, 1.4, -0.5, 0.9, 2.7, 0.3, -1.0, 1.0], 4), ([1.0, 3.0, 3.0, 2.0], 1),
    ([float("nan"), 5.0, 1.0], 0), ([1.0, float("nan"), 5.0, 5.0], 2), ([-float("inf")] * 3, 0)])
def test_argmax_semantics(torch_cuda, pkg, vals, exp):
    torch = torch_cuda
    assert int(pkg.runtime.argmax(_dev(torch, np.array(vals, np.float32))).item()) == exp


def test_argmax_large_matches_oracle(torch_cuda, pkg, oracle):
    torch = torch_cuda
    rng = np.random.default_rng(9)
    v = rng.standard_normal(50257).astype(np.float32)
    v[[17, 40000]] = v.max() + 1                       # tie -> lowest index
    assert int(pkg.runtime.argmax(_dev(torch, v)).item()) == oracle.argmax(v) == 17


def test_silu_gelu_bit_exact(torch_cuda, pkg, oracle):
    torch = torch_cuda
    x = np.linspace(-40, 40, 4001).astype(np.float32)
    u = np.linspace(3, -2, 4001).astype(np.float32)
    h = pkg.runtime.silu_mul(_dev(torch, x), _dev(torch, u)).cpu().numpy()
    assert np.array_equal(h, oracle.silu(x) * u)
    assert np.array_equal(pkg.runtime.gelu(_dev(torch, x)).cpu().numpy(), oracle.gelu(x))


def test_quantizer_bit_exact(torch_cuda, pkg):
    torch = torch_cuda
    rng = np.random.default_rng(2)
    W = (rng.standard_normal((257, 1000)) * 0.02).astype(np.float32)
    W[5] = 0.0
    W[7, :10] = np.float32(2.5) * np.float32(1.0 / 127)
    q, s = pkg.runtime.quantize_rows(_dev(torch, W))
    qr, sr = pkg.pack.quantize_rows(W)
    assert np.array_equal(q.cpu().numpy()[:, :1000], qr) and np.array_equal(s.cpu().numpy(), sr)
    assert (q.cpu().numpy()[:, 1000:] == 0).all()


def test_synthetic_generator_matches_oracle(torch_cuda, pkg, oracle):
    q, s = pkg.runtime.synth_quant_rows(7, 99, 300, 1000, rows=(20, 80), cols=(100, 900))
    qr, sr = oracle.synth_quant(7, 99, 300, 1000, rows=(20, 80), cols=(100, 900))
    assert np.array_equal(q.cpu().numpy()[:, :800], qr) and np.array_equal(s.cpu().numpy(), sr)
