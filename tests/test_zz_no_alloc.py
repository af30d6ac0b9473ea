"""b2_attn_decode_static: decode attention for callers that cannot allocate device
memory (its scratch is a fixed device array inside the library). Collected last
on purpose, so a failure here comes after every other test has run.

The output must equal the workspace-taking b2_attn_decode bit for bit (the same
tolerance as every attention parity test here: exact), on two calls in a row —
the second call reuses the array exactly as the first left it."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("H,KVH,dh,n,max_seq", [(32, 32, 128, 640, 768), (32, 4, 64, 200, 2048),
                                                (4, 2, 16, 7, 32)])
def test_static_scratch_matches_workspace_entry_point(pkg, H, KVH, dh, n, max_seq):
    import torch
    rt = pkg.runtime
    rng = np.random.default_rng(n)
    q = torch.from_numpy((rng.standard_normal(H * dh) * 0.3).astype(np.float32)).cuda()
    K = torch.from_numpy(rng.standard_normal((KVH, max_seq, dh)).astype(np.float32)).cuda()
    V = torch.from_numpy(rng.standard_normal((KVH, max_seq, dh)).astype(np.float32)).cuda()
    ref = rt.attn_decode(q, K, V, H, KVH, dh, n, max_seq).cpu().numpy()
    for _ in range(2):
        got = rt.attn_decode_static(q, K, V, H, KVH, dh, n, max_seq)
        torch.cuda.synchronize()
        assert np.array_equal(got.cpu().numpy(), ref)


def test_static_scratch_rejects_oversized_problem(pkg):
    import torch
    rt = pkg.runtime
    H, KVH, dh, max_seq = 64, 64, 256, 16384          # ~16.9 MB of partials > 4 MiB
    q = torch.zeros(H * dh, device="cuda")
    kv = torch.zeros(1, device="cuda")
    out = torch.zeros(H * dh, device="cuda")
    rc = rt.lib().b2_attn_decode_static(ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(kv.data_ptr()),
                                        ctypes.c_void_p(kv.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                                        H, KVH, dh, 10, max_seq, None)
    assert rc == -1
    assert "static array holds" in rt.last_error()


def test_static_scratch_edge_of_the_array(pkg):
    """32 heads of 128 at max_seq 16128 need 4,193,408 bytes (just under 4 MiB) and
    run; one more 64-key chunk (max_seq 16129: 4,210,048 bytes) is refused."""
    import torch
    rt = pkg.runtime
    H, KVH, dh, n = 32, 32, 128, 300
    assert rt.lib().b2_attn_decode_workspace(H, KVH, dh, 16128) <= 4 << 20
    assert rt.lib().b2_attn_decode_workspace(H, KVH, dh, 16129) > 4 << 20
    rng = np.random.default_rng(3)
    q = torch.from_numpy((rng.standard_normal(H * dh) * 0.3).astype(np.float32)).cuda()
    K = torch.from_numpy(rng.standard_normal((KVH, 16129, dh)).astype(np.float32)).cuda()
    V = torch.from_numpy(rng.standard_normal((KVH, 16129, dh)).astype(np.float32)).cuda()
    Kf, Vf = K[:, :16128].contiguous(), V[:, :16128].contiguous()
    ref = rt.attn_decode(q, Kf, Vf, H, KVH, dh, n, 16128).cpu().numpy()
    got = rt.attn_decode_static(q, Kf, Vf, H, KVH, dh, n, 16128)
    torch.cuda.synchronize()
    assert np.array_equal(got.cpu().numpy(), ref)
    with pytest.raises(rt.B2Error):
        rt.attn_decode_static(q, K, V, H, KVH, dh, n, 16129)
