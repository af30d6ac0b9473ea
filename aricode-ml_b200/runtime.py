"""Host side of the B200 decode path: ctypes over libb2dec.so (include/b2dec.h).

The host loop follows tools/run_decoder.py (prompt ids in, greedy ids out) but
calls the CUDA library in-process instead of spawning the packed binary. There is
no CPU fallback: if libb2dec.so cannot be loaded the import of this module's
functions raises.

Kernel-level helpers (``gemv_i8`` etc.) take torch CUDA tensors only as device
memory and pass raw pointers to the C ABI.
"""
from __future__ import annotations

import ctypes as C
import json
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libb2dec.so"

B2_OK = 0
ERRORS = {-1: "B2_E_INVALID", -2: "B2_E_IO", -3: "B2_E_FORMAT", -4: "B2_E_CUDA", -5: "B2_E_OOM",
          -6: "B2_E_KV_OVERFLOW", -7: "B2_E_UNSUPPORTED", -8: "B2_E_DEVICE", -9: "B2_E_COMM"}


class B2Error(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")
        self.code = code


class KVOverflow(B2Error):
    """Position reached max_seq (the reference's step returns -1 there)."""


_lib = None

vp = C.c_void_p
i32p = C.POINTER(C.c_int32)
f32p = C.POINTER(C.c_float)


def lib():
    """Load libb2dec.so (building it first if sources are newer)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            from . import build as _build
            _build.build()
        _lib = C.CDLL(str(LIB_PATH))
        _declare(_lib)
    return _lib


def _declare(L):
    L.b2_create.argtypes = [C.c_char_p, C.c_char_p, C.c_int, C.POINTER(vp)]
    L.b2_create_synthetic.argtypes = [C.c_char_p, C.c_uint64, C.c_float, C.c_int, C.POINTER(vp)]
    L.b2_create_synthetic_tp.argtypes = [C.c_char_p, C.c_uint64, C.c_float, C.c_int, C.c_int, C.c_int,
                                         C.POINTER(vp)]
    L.b2_create_tp.argtypes = [C.c_char_p, C.c_char_p, C.c_int, C.c_int, C.c_int, C.POINTER(vp)]
    L.b2_tp_handle.argtypes = [vp, C.c_void_p, C.c_int]
    L.b2_tp_connect.argtypes = [vp, C.c_void_p, C.c_int]
    L.b2_destroy.argtypes = [vp]
    L.b2_reset.argtypes = [vp]
    L.b2_step.argtypes = [vp, i32p, C.c_int, i32p, f32p]
    L.b2_prefill.argtypes = [vp, i32p, C.c_int]
    L.b2_generate.argtypes = [vp, i32p, C.c_int, C.c_int, C.c_int32, i32p, C.POINTER(C.c_int)]
    L.b2_set_position.argtypes = [vp, C.c_int, C.c_int32]
    L.b2_decode_async.argtypes = [vp, C.c_int]
    L.b2_fill_kv_synthetic.argtypes = [vp, C.c_int, C.c_uint64]
    L.b2_set_sampling.argtypes = [vp, C.c_int, C.c_int, C.c_double, C.c_uint32]
    L.b2_batch_init.argtypes = [vp, C.c_int, C.c_int]
    L.b2_batch_reset.argtypes = [vp]
    L.b2_batch_prefill.argtypes = [vp, C.c_int, i32p, C.c_int]
    L.b2_batch_step.argtypes = [vp, i32p, i32p, f32p]
    L.b2_batch_decode_async.argtypes = [vp, C.c_int]
    L.b2_batch_read_output.argtypes = [vp, i32p, C.c_int, C.POINTER(C.c_int)]
    L.b2_batch_generate.argtypes = [vp, i32p, C.c_int, C.c_int, i32p]
    L.b2_sync.argtypes = [vp]
    L.b2_read_output.argtypes = [vp, i32p, C.c_int, C.POINTER(C.c_int)]
    L.b2_set_stream.argtypes = [vp, vp]
    L.b2_query.argtypes = [vp, C.c_char_p, C.POINTER(C.c_double)]
    L.b2_last_error.argtypes = [vp, C.c_char_p, C.c_int]
    L.b2_gemv_i8_rowscale.argtypes = [vp, C.c_int64, vp, vp, vp, vp, C.c_int, C.c_int, vp]
    L.b2_gemv_f32.argtypes = [vp, C.c_int64, vp, vp, vp, C.c_int, C.c_int, vp]
    L.b2_gemv_i4_rowscale.argtypes = [vp, C.c_int64, vp, vp, vp, vp, C.c_int, C.c_int, vp]
    L.b2_gemm_i8_rowscale_workspace.restype = C.c_size_t
    L.b2_gemm_i8_rowscale_workspace.argtypes = [C.c_int, C.c_int64]
    L.b2_gemm_i8_rowscale.argtypes = [vp, C.c_int64, vp, vp, C.c_int64, vp, vp, C.c_int64, C.c_int, C.c_int,
                                      C.c_int, vp, C.c_size_t, vp]
    L.b2_rmsnorm.argtypes = [vp, vp, vp, C.c_int, C.c_float, vp]
    L.b2_layernorm.argtypes = [vp, vp, vp, vp, C.c_int, C.c_float, vp]
    L.b2_rope_apply.argtypes = [vp, vp, C.c_int, C.c_int, C.c_int, vp]
    L.b2_attn_decode_workspace.restype = C.c_size_t
    L.b2_attn_decode_workspace.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int]
    L.b2_attn_decode.argtypes = [vp, vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, vp,
                                 C.c_size_t, vp]
    L.b2_attn_decode_static.argtypes = [vp, vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int,
                                        C.c_int, vp]
    L.b2_argmax.argtypes = [vp, C.c_int64, vp, vp]
    L.b2_silu_mul.argtypes = [vp, vp, vp, C.c_int, vp]
    L.b2_gelu.argtypes = [vp, vp, C.c_int, vp]
    L.b2_quantize_rows.argtypes = [vp, C.c_int64, C.c_int64, vp, C.c_int64, vp, vp]
    L.b2_synth_quant_rows.argtypes = [C.c_uint64, C.c_uint64, C.c_int64, C.c_float, C.c_int64,
                                      C.c_int64, C.c_int64, C.c_int64, vp, C.c_int64, vp, vp]
    L.b2_synth_fill_f32.argtypes = [C.c_uint64, C.c_uint64, C.c_int64, C.c_int64, C.c_float, vp, vp]


def last_error(ctx=None):
    buf = C.create_string_buffer(1024)
    lib().b2_last_error(ctx, buf, 1024)
    return buf.value.decode(errors="replace")


def check(code, ctx=None):
    if code != B2_OK:
        msg = last_error(ctx)
        if code == -6:
            raise KVOverflow(code, msg)
        raise B2Error(code, msg)


def parse_sample(spec):
    """--sample spec -> (mode, top_k, temperature): 'greedy', 'temperature:T' or
    'topk:K:T' (the reference's parse_sample_spec, aricode_pack.py:2035-2065)."""
    parts = str(spec).split(":")
    try:
        if parts[0] == "greedy" and len(parts) == 1:
            return 0, 0, 0.0
        if parts[0] == "temperature" and len(parts) == 2:
            return 1, 0, float(parts[1])
        if parts[0] == "topk" and len(parts) == 3:
            return 2, int(parts[1]), float(parts[2])
    except ValueError:
        pass
    raise ValueError(f"--sample expects greedy, temperature:T or topk:K:T; got {spec!r}")


def fnv1a64(name: str) -> int:
    """Tensor id of a synthetic tensor (same hash as the C++ runtime)."""
    h = 0xcbf29ce484222325
    for c in name.encode():
        h ^= c
        h = (h * 0x100000001b3) & 0xFFFFFFFFFFFFFFFF
    return h


def _i32(seq):
    arr = (C.c_int32 * max(len(seq), 1))(*[int(t) for t in seq])
    return arr


def tp_gather_handles(handle, rank, size, exchange):
    """Every rank's 64-byte exchange-buffer handle, concatenated in rank order (the
    b2_tp_connect argument). `exchange(handle)` returns the list of all ranks'
    handles in rank order; this rank's own must come back in its slot."""
    if len(handle) != 64:
        raise ValueError("a handle is 64 bytes")
    handles = list(exchange(bytes(handle)))
    if len(handles) != size or any(len(b) != 64 for b in handles):
        raise ValueError("exchange must return one 64-byte handle per rank")
    if handles[rank] != bytes(handle):
        raise ValueError("exchange returned the handles out of rank order")
    return b"".join(handles)


class Decoder:
    """One model on one GPU. ``Decoder(blob_path)`` or ``Decoder.synthetic(plan, seed)``."""

    def __init__(self, blob_path=None, plan=None, device=0, *, _ctx=None):
        self._ctx = vp()
        if _ctx is not None:
            self._ctx = _ctx
        else:
            plan_s = json.dumps(plan).encode() if plan is not None else None
            check(lib().b2_create(str(blob_path).encode(), plan_s, int(device), C.byref(self._ctx)))
        self.vocab = int(self.query("vocab"))
        self.max_seq = int(self.query("max_seq"))

    @classmethod
    def synthetic(cls, plan, seed=0, stdv=0.02, device=0):
        ctx = vp()
        check(lib().b2_create_synthetic(json.dumps(plan).encode(), int(seed), float(stdv),
                                        int(device), C.byref(ctx)))
        return cls(_ctx=ctx)

    @classmethod
    def synthetic_tp(cls, plan, rank, size, exchange, seed=0, stdv=0.02, device=0):
        """Rank `rank` of a tensor-parallel decoder over `size` GPUs (one process
        per GPU). `exchange(handle_bytes) -> list of every rank's bytes, in rank
        order` moves the 64-byte buffer handles between the processes (for example
        torch.distributed.all_gather_object). Every rank must then call the same
        methods in the same order."""
        ctx = vp()
        check(lib().b2_create_synthetic_tp(json.dumps(plan).encode(), int(seed), float(stdv), int(device),
                                           int(rank), int(size), C.byref(ctx)))
        return cls(_ctx=ctx)._connect(rank, size, exchange)

    @classmethod
    def from_blob_tp(cls, blob_path, rank, size, exchange, device=0, plan=None):
        """Rank `rank` of a tensor-parallel decoder over `size` GPUs from a packed
        blob (each rank loads its rows); `exchange` as for synthetic_tp."""
        ctx = vp()
        plan_s = json.dumps(plan).encode() if plan is not None else None
        check(lib().b2_create_tp(str(blob_path).encode(), plan_s, int(device), int(rank), int(size),
                                 C.byref(ctx)))
        return cls(_ctx=ctx)._connect(rank, size, exchange)

    def _connect(self, rank, size, exchange):
        dec, ctx = self, self._ctx
        if size > 1:
            h = C.create_string_buffer(64)
            dec._ck(lib().b2_tp_handle(ctx, h, 64))
            joined = tp_gather_handles(h.raw, rank, size, exchange)
            allh = C.create_string_buffer(joined, 64 * size)
            dec._ck(lib().b2_tp_connect(ctx, allh, 64 * size))
            # graph capture in b2_tp_connect takes each rank its own time: meet once
            # more, so that the first step's cross-rank waits (bounded at about 1 s)
            # do not start seconds apart
            exchange(bytes(64))
        return dec

    def close(self):
        if self._ctx:
            lib().b2_destroy(self._ctx)
            self._ctx = vp()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def _ck(self, code):
        check(code, self._ctx)

    def query(self, key):
        v = C.c_double()
        self._ck(lib().b2_query(self._ctx, key.encode(), C.byref(v)))
        return v.value

    def reset(self):
        self._ck(lib().b2_reset(self._ctx))

    def step(self, tok, want_logits=False):
        """One token: returns (next_id, logits or None)."""
        import numpy as np
        t = (C.c_int32 * 1)(int(tok))
        nxt = (C.c_int32 * 1)()
        logits = np.zeros(self.vocab, np.float32) if want_logits else None
        self._ck(lib().b2_step(self._ctx, t, 1, nxt,
                               logits.ctypes.data_as(f32p) if want_logits else None))
        return int(nxt[0]), logits

    def prefill(self, toks):
        a = _i32(toks)
        self._ck(lib().b2_prefill(self._ctx, a, len(toks)))

    def generate(self, prompt, max_new, eos=-1):
        """Greedy generation (reference loop semantics); returns the generated ids."""
        p = _i32(prompt)
        out = (C.c_int32 * max(max_new, 1))()
        n = C.c_int(0)
        self._ck(lib().b2_generate(self._ctx, p, len(prompt), int(max_new), int(eos), out,
                                   C.byref(n)))
        return list(out[:n.value])

    def set_position(self, pos, next_tok):
        self._ck(lib().b2_set_position(self._ctx, int(pos), int(next_tok)))

    def set_sampling(self, sample="greedy", seed=20260502):
        """--sample spec (greedy | temperature:T | topk:K:T) and the LCG seed."""
        mode, k, temp = parse_sample(sample)
        self._ck(lib().b2_set_sampling(self._ctx, mode, k, temp, int(seed) & 0xFFFFFFFF))

    # ---- batched decode (n_seq sequences, one token each per step)
    def batch_init(self, n_seq, max_steps=256):
        self._ck(lib().b2_batch_init(self._ctx, int(n_seq), int(max_steps)))
        self.n_seq = int(n_seq)

    def batch_reset(self):
        self._ck(lib().b2_batch_reset(self._ctx))

    def batch_prefill(self, seq, toks):
        self._ck(lib().b2_batch_prefill(self._ctx, int(seq), _i32(toks), len(toks)))

    def batch_step(self, toks, want_logits=False):
        """One token per sequence: returns (next ids, logits [n_seq, vocab] or None)."""
        import numpy as np
        nxt = (C.c_int32 * self.n_seq)()
        logits = np.zeros((self.n_seq, self.vocab), np.float32) if want_logits else None
        self._ck(lib().b2_batch_step(self._ctx, _i32(toks), nxt,
                                     logits.ctypes.data_as(f32p) if want_logits else None))
        return list(nxt), logits

    def batch_decode_async(self, n_steps):
        self._ck(lib().b2_batch_decode_async(self._ctx, int(n_steps)))

    def batch_read_output(self, max_steps):
        import numpy as np
        out = np.zeros((max_steps, self.n_seq), np.int32)
        n = C.c_int(0)
        self._ck(lib().b2_batch_read_output(self._ctx, out.ctypes.data_as(i32p), int(max_steps), C.byref(n)))
        return out[: n.value]

    def batch_generate(self, prompts, max_new):
        """prompts [n_seq][P] (equal lengths) -> generated ids [n_seq][max_new]."""
        import numpy as np
        p = np.ascontiguousarray(prompts, np.int32)
        out = np.zeros((p.shape[0], max_new), np.int32)
        self._ck(lib().b2_batch_generate(self._ctx, p.ctypes.data_as(i32p), p.shape[1], int(max_new),
                                         out.ctypes.data_as(i32p)))
        return out

    def fill_kv_synthetic(self, count, seed=0):
        """KV rows [0, count) from the synthetic generator (the oracle's fill_kv) and
        the position set to count: decoding can start mid-sequence without a prefill."""
        self._ck(lib().b2_fill_kv_synthetic(self._ctx, int(count), int(seed)))

    def decode_async(self, n_steps):
        self._ck(lib().b2_decode_async(self._ctx, int(n_steps)))

    def sync(self):
        self._ck(lib().b2_sync(self._ctx))

    def read_output(self, max_ids=None):
        max_ids = max_ids or self.max_seq
        out = (C.c_int32 * max_ids)()
        n = C.c_int(0)
        self._ck(lib().b2_read_output(self._ctx, out, max_ids, C.byref(n)))
        return list(out[:n.value])

    def set_stream(self, stream_handle):
        self._ck(lib().b2_set_stream(self._ctx, vp(int(stream_handle))))


# ----------------------------------------------------------------- kernel-level helpers
def _ptr(t):
    return vp(t.data_ptr()) if t is not None else None


def _stream(stream):
    if stream is None:
        import torch
        return vp(torch.cuda.current_stream().cuda_stream)
    return vp(int(stream))


def gemv_i8(W, scale, x, bias=None, y=None, n=None, stream=None):
    """W: int8 [m, ld] CUDA tensor (ld % 16 == 0, zero padded), returns y [m]."""
    import torch
    m, ld = W.shape
    n = n or ld
    y = y if y is not None else torch.empty(m, dtype=torch.float32, device=W.device)
    check(lib().b2_gemv_i8_rowscale(_ptr(W), ld, _ptr(scale), _ptr(x), _ptr(bias), _ptr(y), m, n,
                                    _stream(stream)))
    return y


def gemv_i4(W, scale, x, n, bias=None, y=None, stream=None):
    """W: uint8 [m, ld] packed int4 CUDA tensor (ld % 16 == 0), n codes per row."""
    import torch
    m, ld = W.shape
    y = y if y is not None else torch.empty(m, dtype=torch.float32, device=W.device)
    check(lib().b2_gemv_i4_rowscale(_ptr(W), ld, _ptr(scale), _ptr(x), _ptr(bias), _ptr(y), m, n, _stream(stream)))
    return y


def gemm_i8(W, scale, X, bias=None, n=None, stream=None):
    """T vectors at once on the tensor cores: X [T, n] f32 -> Y [T, m]; W int8 [m, ld]."""
    import torch
    m, ld = W.shape
    T = X.shape[0]
    n = n or ld
    Y = torch.empty(T, m, dtype=torch.float32, device=W.device)
    nb = lib().b2_gemm_i8_rowscale_workspace(T, ld)
    ws = torch.empty(nb, dtype=torch.uint8, device=W.device)
    check(lib().b2_gemm_i8_rowscale(_ptr(W), ld, _ptr(scale), _ptr(X), X.stride(0), _ptr(bias), _ptr(Y), m, m, n, T,
                                    _ptr(ws), nb, _stream(stream)))
    return Y


def gemv_f32(W, x, bias=None, y=None, n=None, stream=None):
    import torch
    m, ld = W.shape
    n = n or ld
    y = y if y is not None else torch.empty(m, dtype=torch.float32, device=W.device)
    check(lib().b2_gemv_f32(_ptr(W), ld, _ptr(x), _ptr(bias), _ptr(y), m, n, _stream(stream)))
    return y


def rmsnorm(x, g, eps=1e-5, stream=None):
    import torch
    y = torch.empty_like(x)
    check(lib().b2_rmsnorm(_ptr(x), _ptr(g), _ptr(y), x.numel(), eps, _stream(stream)))
    return y


def layernorm(x, g, b, eps=1e-5, stream=None):
    import torch
    y = torch.empty_like(x)
    check(lib().b2_layernorm(_ptr(x), _ptr(g), _ptr(b), _ptr(y), x.numel(), eps, _stream(stream)))
    return y


def rope_apply(v, table, pos, d_head, stream=None):
    check(lib().b2_rope_apply(_ptr(v), _ptr(table), int(pos), int(d_head), v.numel() // d_head,
                              _stream(stream)))
    return v


def attn_workspace_bytes(n_heads, n_kv_heads, d_head, max_seq):
    return int(lib().b2_attn_decode_workspace(n_heads, n_kv_heads, d_head, max_seq))


def attn_decode(q, K, V, n_heads, n_kv_heads, d_head, n, max_seq, workspace=None, out=None,
                stream=None):
    import torch
    ws_bytes = attn_workspace_bytes(n_heads, n_kv_heads, d_head, max_seq)
    if workspace is None:
        workspace = torch.zeros(ws_bytes, dtype=torch.uint8, device=q.device)
    if out is None:
        out = torch.empty(n_heads * d_head, dtype=torch.float32, device=q.device)
    check(lib().b2_attn_decode(_ptr(q), _ptr(K), _ptr(V), _ptr(out), n_heads, n_kv_heads, d_head,
                               int(n), int(max_seq), _ptr(workspace), workspace.numel(),
                               _stream(stream)))
    return out


def attn_decode_static(q, K, V, n_heads, n_kv_heads, d_head, n, max_seq, stream=None):
    """b2_attn_decode with the library's fixed device scratch (no workspace, no
    allocation inside the call; the output tensor is the caller's)."""
    import torch
    out = torch.empty(n_heads * d_head, dtype=torch.float32, device=q.device)
    check(lib().b2_attn_decode_static(_ptr(q), _ptr(K), _ptr(V), _ptr(out), n_heads, n_kv_heads,
                                      d_head, int(n), int(max_seq), _stream(stream)))
    return out


def argmax(v, stream=None):
    import torch
    out = torch.empty(1, dtype=torch.int32, device=v.device)
    check(lib().b2_argmax(_ptr(v), v.numel(), _ptr(out), _stream(stream)))
    return out


def silu_mul(g, u, stream=None):
    import torch
    h = torch.empty_like(g)
    check(lib().b2_silu_mul(_ptr(g), _ptr(u), _ptr(h), g.numel(), _stream(stream)))
    return h


def gelu(x, stream=None):
    import torch
    y = torch.empty_like(x)
    check(lib().b2_gelu(_ptr(x), _ptr(y), x.numel(), _stream(stream)))
    return y


def quantize_rows(W, ldq=None, stream=None):
    import torch
    m, n = W.shape
    ldq = ldq or (n + 15) // 16 * 16
    q = torch.empty((m, ldq), dtype=torch.int8, device=W.device)
    s = torch.empty(m, dtype=torch.float32, device=W.device)
    check(lib().b2_quantize_rows(_ptr(W), m, n, _ptr(q), ldq, _ptr(s), _stream(stream)))
    return q, s


def synth_quant_rows(seed, tensor_id, m, n, stdv=0.02, rows=None, cols=None, device="cuda",
                     stream=None):
    import torch
    r0, r1 = rows or (0, m)
    c0, c1 = cols or (0, n)
    w = c1 - c0
    ldq = (w + 15) // 16 * 16
    q = torch.empty((r1 - r0, ldq), dtype=torch.int8, device=device)
    s = torch.empty(r1 - r0, dtype=torch.float32, device=device)
    check(lib().b2_synth_quant_rows(seed, tensor_id, n, stdv, r0, r1, c0, c1, _ptr(q), ldq, _ptr(s),
                                    _stream(stream)))
    return q, s
