"""ctypes wrapper of the CPU oracle (oracle/refdec.c).

TEST INFRASTRUCTURE: imported only by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, as the checker / timed CPU baseline. The product
path never imports this module.

``OracleModel(plan, tensors)`` takes the same launch plan and tensors the CUDA
runtime consumes (``aricode-ml_b200.blob.read_blob`` output, or tensors built in
memory) and runs the restated reference decode loop on the host.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"


def build(force=False):
    """Compile the oracle with its Makefile (gcc, seconds)."""
    if force or not LIB_PATH.exists() or \
            LIB_PATH.stat().st_mtime < max((HERE / f).stat().st_mtime
                                           for f in ("refdec.c", "refdec.h", "Makefile")):
        subprocess.run(["make", "-C", str(HERE), "-s"], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = C.CDLL(str(LIB_PATH))
        _declare(_lib)
    return _lib


f32p = C.POINTER(C.c_float)
i8p = C.POINTER(C.c_int8)
i32p = C.POINTER(C.c_int32)


class Mat(C.Structure):
    _fields_ = [("is_i8", C.c_int), ("w", C.c_void_p), ("s", f32p), ("ld", C.c_int64)]


class Block(C.Structure):
    _fields_ = [("type", C.c_int), ("norm", C.c_int), ("ng", f32p), ("nb", f32p),
                ("rope", C.c_int), ("n_heads", C.c_int), ("n_kv_heads", C.c_int),
                ("d_head", C.c_int), ("kv_slot", C.c_int),
                ("q", Mat), ("k", Mat), ("v", Mat), ("o", Mat),
                ("bq", f32p), ("bk", f32p), ("bv", f32p), ("bo", f32p),
                ("ffn_kind", C.c_int), ("d_ffn", C.c_int),
                ("w1", Mat), ("w3", Mat), ("w2", Mat), ("b1", f32p), ("b2", f32p)]


class Model(C.Structure):
    _fields_ = [("vocab", C.c_int), ("d", C.c_int), ("max_seq", C.c_int),
                ("n_blocks", C.c_int), ("n_kv_slots", C.c_int), ("eps", C.c_float),
                ("emb", Mat), ("pos", f32p), ("max_pos", C.c_int),
                ("blocks", C.POINTER(Block)),
                ("fn_kind", C.c_int), ("fn_g", f32p), ("fn_b", f32p),
                ("lm", Mat), ("lm_b", f32p), ("rope", f32p),
                ("max_heads", C.c_int), ("max_kv_dim", C.c_int), ("max_ffn", C.c_int)]


class State(C.Structure):
    _fields_ = [("K", C.POINTER(f32p)), ("V", C.POINTER(f32p)), ("kv_elems", C.POINTER(C.c_size_t)),
                ("n_slots", C.c_int), ("count", C.c_int),
                ("x", f32p), ("h", f32p), ("q", f32p), ("k", f32p), ("v", f32p),
                ("att", f32p), ("f1", f32p), ("f3", f32p), ("logits", f32p)]


def _declare(L):
    L.b2o_exp_f.restype = C.c_float; L.b2o_exp_f.argtypes = [C.c_float]
    L.b2o_exp_d.restype = C.c_double; L.b2o_exp_d.argtypes = [C.c_double]
    L.b2o_silu.restype = C.c_float; L.b2o_silu.argtypes = [C.c_float]
    L.b2o_gelu.restype = C.c_float; L.b2o_gelu.argtypes = [C.c_float]
    L.b2o_quantize_rows.argtypes = [f32p, C.c_int64, C.c_int64, i8p, C.c_int64, f32p]
    L.b2o_gemv_i4.argtypes = [C.c_void_p, C.c_int64, f32p, f32p, C.c_int64, C.c_int64, f32p]
    L.b2o_unpack_i4.argtypes = [C.c_void_p, C.c_int64, i8p]
    L.b2o_gemv_i8.argtypes = [i8p, C.c_int64, f32p, f32p, C.c_int64, C.c_int64, f32p]
    L.b2o_gemv_f32.argtypes = [f32p, C.c_int64, f32p, C.c_int64, C.c_int64, f32p]
    L.b2o_rmsnorm.argtypes = [f32p, f32p, C.c_int, C.c_float, f32p]
    L.b2o_layernorm.argtypes = [f32p, f32p, f32p, C.c_int, C.c_float, f32p]
    L.b2o_rope_table.argtypes = [C.c_int, C.c_int, C.c_double, f32p]
    L.b2o_rope_apply.argtypes = [f32p, f32p, C.c_int, C.c_int]
    L.b2o_attn_decode.argtypes = [f32p, f32p, f32p, C.c_int, C.c_int, C.c_int, C.c_int,
                                  C.c_int, f32p]
    L.b2o_argmax.restype = C.c_int32; L.b2o_argmax.argtypes = [f32p, C.c_int64]
    L.b2o_synth_value.restype = C.c_float
    L.b2o_synth_value.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64, C.c_float]
    L.b2o_synth_fill_f32.argtypes = [C.c_uint64, C.c_uint64, C.c_int64, C.c_int64, C.c_float, f32p]
    L.b2o_synth_quant_rows.argtypes = [C.c_uint64, C.c_uint64, C.c_int64, C.c_float, C.c_int64,
                                       C.c_int64, C.c_int64, C.c_int64, i8p, C.c_int64, f32p]
    L.b2o_state_init.restype = C.c_int
    L.b2o_state_init.argtypes = [C.POINTER(Model), C.POINTER(State)]
    L.b2o_state_free.argtypes = [C.POINTER(State)]
    L.b2o_state_reset.argtypes = [C.POINTER(Model), C.POINTER(State)]
    L.b2o_step.restype = C.c_int32
    L.b2o_step.argtypes = [C.POINTER(Model), C.POINTER(State), C.c_int32, f32p, C.c_int]
    L.b2o_generate.restype = C.c_int
    L.b2o_generate.argtypes = [C.POINTER(Model), C.POINTER(State), i32p, C.c_int, C.c_int, i32p]
    L.b2o_state_fill_kv.argtypes = [C.POINTER(Model), C.POINTER(State), C.c_int, C.c_uint64]
    L.b2o_set_threads.argtypes = [C.c_int]
    L.b2o_get_threads.restype = C.c_int
    L.b2o_lcg_next.restype = C.c_uint32; L.b2o_lcg_next.argtypes = [C.c_uint32]
    L.b2o_topk_filter.argtypes = [f32p, C.c_int64, C.c_int]
    L.b2o_sample_temperature.restype = C.c_int32
    L.b2o_sample_temperature.argtypes = [f32p, C.c_int64, C.c_double, C.c_double]
    L.b2o_sample.restype = C.c_int32
    L.b2o_sample.argtypes = [f32p, C.c_int64, C.c_int, C.c_int, C.c_double, C.POINTER(C.c_uint32)]
    L.b2o_generate_ex.restype = C.c_int
    L.b2o_generate_ex.argtypes = [C.POINTER(Model), C.POINTER(State), i32p, C.c_int, C.c_int, C.c_int32,
                                  C.c_int, C.c_int, C.c_double, C.c_uint32, i32p]
    L.b2o_set_matvec_mode.argtypes = [C.c_int]
    L.b2o_get_matvec_mode.restype = C.c_int
    L.b2o_dot_i8_f32acc.restype = C.c_float
    L.b2o_dot_i8_f32acc.argtypes = [i8p, f32p, C.c_int64]
    L.b2o_dot_i8_f64.restype = C.c_double
    L.b2o_dot_i8_f64.argtypes = [i8p, f32p, C.c_int64]


def _p(a, t=f32p):
    return a.ctypes.data_as(t) if a is not None else None


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


# ------------------------------------------------------------------ kernels (numpy in/out)
def set_threads(n):
    lib().b2o_set_threads(int(n))


MATVEC_EXACT, MATVEC_F32ACC, MATVEC_F64 = 0, 1, 2


class matvec_mode:
    """Context manager: the int8 matvec the oracle uses inside the block —
    MATVEC_EXACT (fixed-point dot, the GPU's bits), MATVEC_F32ACC (8-lane f32 FMA
    accumulation, the reference builtin as README.md:128-131 describes it) or
    MATVEC_F64 (f64 accumulation, the truth model for the matvec)."""

    def __init__(self, mode):
        self.mode = mode

    def __enter__(self):
        self.old = lib().b2o_get_matvec_mode()
        lib().b2o_set_matvec_mode(self.mode)
        return self

    def __exit__(self, *exc):
        lib().b2o_set_matvec_mode(self.old)
        return False


def dot_i8_f32acc(w, x):
    w = _c(w, np.int8); x = _c(x, np.float32)
    return np.float32(lib().b2o_dot_i8_f32acc(_p(w, i8p), _p(x), w.size))


def dot_i8_f64(w, x):
    w = _c(w, np.int8); x = _c(x, np.float32)
    return lib().b2o_dot_i8_f64(_p(w, i8p), _p(x), w.size)


def exp_f(x):
    return np.float32(lib().b2o_exp_f(float(x)))


def exp_d(x):
    return lib().b2o_exp_d(float(x))


def silu(x):
    return np.array([lib().b2o_silu(float(v)) for v in np.ravel(x)], np.float32).reshape(np.shape(x))


def gelu(x):
    return np.array([lib().b2o_gelu(float(v)) for v in np.ravel(x)], np.float32).reshape(np.shape(x))


def quantize_rows(W):
    W = _c(W, np.float32)
    m, n = W.shape
    q = np.zeros((m, n), np.int8)
    s = np.zeros(m, np.float32)
    lib().b2o_quantize_rows(_p(W), m, n, _p(q, i8p), n, _p(s))
    return q, s


def gemv_i8(q, scale, x):
    """q: [m, n] int8 (any row stride is re-packed), scale [m], x [n] -> y [m]."""
    q = _c(q, np.int8); scale = _c(scale, np.float32); x = _c(x, np.float32)
    m, n = q.shape
    y = np.zeros(m, np.float32)
    lib().b2o_gemv_i8(_p(q, i8p), n, _p(scale), _p(x), m, n, _p(y))
    return y


def gemv_i4(packed, scale, x, n):
    """packed: uint8 [m, ld] (two codes a byte, even column low), n logical columns."""
    packed = _c(packed, np.uint8); scale = _c(scale, np.float32); x = _c(x, np.float32)
    m, ld = packed.shape
    y = np.zeros(m, np.float32)
    lib().b2o_gemv_i4(packed.ctypes.data, ld, _p(scale), _p(x), m, n, _p(y))
    return y


def unpack_i4(packed, n):
    packed = _c(packed, np.uint8).ravel()
    out = np.zeros(n, np.int8)
    lib().b2o_unpack_i4(packed.ctypes.data, n, _p(out, i8p))
    return out


def gemv_f32(W, x):
    W = _c(W, np.float32); x = _c(x, np.float32)
    m, n = W.shape
    y = np.zeros(m, np.float32)
    lib().b2o_gemv_f32(_p(W), n, _p(x), m, n, _p(y))
    return y


def rmsnorm(x, g, eps=1e-5):
    x = _c(x, np.float32); g = _c(g, np.float32)
    y = np.zeros_like(x)
    lib().b2o_rmsnorm(_p(x), _p(g), x.size, eps, _p(y))
    return y


def layernorm(x, g, b, eps=1e-5):
    x = _c(x, np.float32); g = _c(g, np.float32); b = _c(b, np.float32)
    y = np.zeros_like(x)
    lib().b2o_layernorm(_p(x), _p(g), _p(b), x.size, eps, _p(y))
    return y


def rope_table(max_seq, d_head, theta):
    t = np.zeros((max_seq, d_head), np.float32)
    lib().b2o_rope_table(max_seq, d_head, float(theta), _p(t))
    return t


def rope_apply(v, table, pos):
    v = _c(v, np.float32).copy(); table = _c(table, np.float32)
    lib().b2o_rope_apply(_p(v), _p(table), pos, v.size)
    return v


def attn_decode(q, K, V, n_heads, n_kv_heads, d_head, n, max_seq):
    q = _c(q, np.float32); K = _c(K, np.float32); V = _c(V, np.float32)
    out = np.zeros(n_heads * d_head, np.float32)
    lib().b2o_attn_decode(_p(q), _p(K), _p(V), n_heads, n_kv_heads, d_head, n, max_seq, _p(out))
    return out


SAMPLE_GREEDY, SAMPLE_TEMPERATURE, SAMPLE_TOPK = 0, 1, 2


def parse_sample(spec):
    """--sample spec -> (mode, top_k, temperature): greedy | temperature:T | topk:K:T
    (aricode_pack.py:2035-2065)."""
    parts = spec.split(":")
    if parts[0] == "greedy" and len(parts) == 1:
        return SAMPLE_GREEDY, 0, 0.0
    if parts[0] == "temperature" and len(parts) == 2:
        return SAMPLE_TEMPERATURE, 0, float(parts[1])
    if parts[0] == "topk" and len(parts) == 3:
        return SAMPLE_TOPK, int(parts[1]), float(parts[2])
    raise ValueError(f"bad --sample spec {spec!r}")


def lcg_next(state):
    return int(lib().b2o_lcg_next(state & 0xFFFFFFFF))


def topk_filter(v, k):
    v = _c(v, np.float32).copy()
    lib().b2o_topk_filter(_p(v), v.size, int(k))
    return v


def sample_temperature(v, temperature, unit):
    v = _c(v, np.float32).copy()
    return int(lib().b2o_sample_temperature(_p(v), v.size, float(temperature), float(unit))), v


def argmax(v):
    v = _c(v, np.float32)
    return int(lib().b2o_argmax(_p(v), v.size))


def synth_f32(seed, tensor_id, m, n, stdv=0.02):
    out = np.zeros((m, n), np.float32)
    lib().b2o_synth_fill_f32(seed, tensor_id, m, n, stdv, _p(out))
    return out


def synth_quant(seed, tensor_id, m, n, stdv=0.02, rows=None, cols=None):
    r0, r1 = rows if rows else (0, m)
    c0, c1 = cols if cols else (0, n)
    q = np.zeros((r1 - r0, c1 - c0), np.int8)
    s = np.zeros(r1 - r0, np.float32)
    lib().b2o_synth_quant_rows(seed, tensor_id, n, stdv, r0, r1, c0, c1, _p(q, i8p),
                               c1 - c0, _p(s))
    return q, s


# ------------------------------------------------------------------ whole decoder
class OracleModel:
    """Host-side decoder over a launch plan and its tensors (read_blob output)."""

    def __init__(self, plan, tensors, threads=1):
        self.plan = plan
        self.keep = []               # numpy arrays the C structs point into
        t = {k: v for k, v in tensors.items()}
        self.threads = threads

        def arr(name, dt=np.float32):
            a = np.ascontiguousarray(t[name], dtype=dt)
            self.keep.append(a)
            return a

        def mat(name):
            w = t[name]
            if w.dtype == np.uint8:                      # int4, packed two codes per byte
                a = arr(name, np.uint8)
                s = arr(name + "_scales")
                return Mat(2, a.ctypes.data, _p(s), a.shape[1])
            if w.dtype == np.int8:
                a = arr(name, np.int8)
                s = arr(name + "_scales")
                return Mat(1, a.ctypes.data, _p(s), a.shape[1])
            a = arr(name)
            return Mat(0, a.ctypes.data, None, a.shape[1])

        def vec(name):
            return _p(arr(name)) if name else None

        blocks = (Block * len(plan["blocks"]))()
        slot = 0
        max_heads = max_kv = max_ffn = 1
        rope_dh, rope_theta = None, None
        for i, b in enumerate(plan["blocks"]):
            B = blocks[i]
            B.type = 0 if b["type"] == "attn" else 1
            B.norm = 0 if b["norm"]["kind"] == "rms" else 1
            B.ng = vec(b["norm"]["g"])
            B.nb = vec(b["norm"].get("b"))
            if b["type"] == "attn":
                B.rope = 1 if b["rope"] else 0
                B.n_heads, B.n_kv_heads, B.d_head = b["n_heads"], b["n_kv_heads"], b["d_head"]
                B.kv_slot = slot; slot += 1
                B.q, B.k, B.v, B.o = mat(b["q"]), mat(b["k"]), mat(b["v"]), mat(b["o"])
                bias = b.get("bias") or {}
                B.bq, B.bk, B.bv, B.bo = (vec(bias.get(p)) for p in "qkvo")
                max_heads = max(max_heads, b["n_heads"] * b["d_head"])
                max_kv = max(max_kv, b["n_kv_heads"] * b["d_head"])
                if b["rope"]:
                    if rope_dh not in (None, b["d_head"]) or rope_theta not in (None, b["theta"]):
                        raise ValueError("RoPE sub-blocks must share d_head and theta")
                    rope_dh, rope_theta = b["d_head"], b["theta"]
            else:
                B.d_ffn = b["d_ffn"]
                max_ffn = max(max_ffn, b["d_ffn"])
                if b["kind"] == "swiglu":
                    B.ffn_kind = 0
                    B.w1, B.w3, B.w2 = mat(b["gate"]), mat(b["up"]), mat(b["down"])
                else:
                    B.ffn_kind = 1
                    B.w1, B.w2 = mat(b["fc1"]), mat(b["fc2"])
                    B.b1, B.b2 = vec(b["fc1_b"]), vec(b["fc2_b"])
        self.blocks = blocks
        M = Model()
        M.vocab, M.d, M.max_seq = plan["vocab"], plan["d_model"], plan["max_seq"]
        M.n_blocks, M.n_kv_slots, M.eps = len(plan["blocks"]), slot, plan.get("eps", 1e-5)
        M.emb = mat(plan["embedding"])
        M.pos = vec(plan.get("pos_embedding"))
        M.max_pos = plan.get("max_pos", 0)
        M.blocks = C.cast(blocks, C.POINTER(Block))
        fn = plan["final_norm"]
        M.fn_kind = 0 if fn["kind"] == "rms" else 1
        M.fn_g, M.fn_b = vec(fn["g"]), vec(fn.get("b"))
        M.lm = mat(plan["lm_head"]["W"])
        M.lm_b = vec(plan["lm_head"]["b"])
        if rope_dh is not None:
            self.rope = rope_table(plan["max_seq"], rope_dh, rope_theta)
            M.rope = _p(self.rope)
        M.max_heads, M.max_kv_dim, M.max_ffn = max_heads, max_kv, max_ffn
        self.model = M
        self.state = State()
        if lib().b2o_state_init(C.byref(M), C.byref(self.state)) != 0:
            raise MemoryError("oracle state allocation failed")

    def __del__(self):
        try:
            lib().b2o_state_free(C.byref(self.state))
        except Exception:
            pass

    @property
    def count(self):
        return self.state.count

    def reset(self):
        lib().b2o_state_reset(C.byref(self.model), C.byref(self.state))

    def fill_kv(self, count, seed=0):
        """Synthetic KV rows [0, count) and position = count (benchmark sampling)."""
        lib().b2o_state_fill_kv(C.byref(self.model), C.byref(self.state), int(count), int(seed))

    def step(self, tok, want_logits=True):
        """Returns (next_id, logits) — next_id -1 on KV overflow."""
        set_threads(self.threads)
        logits = np.zeros(self.plan["vocab"], np.float32) if want_logits else None
        r = lib().b2o_step(C.byref(self.model), C.byref(self.state), int(tok),
                           _p(logits) if want_logits else None, 1 if want_logits else 0)
        return int(r), logits

    def generate_sampled(self, prompt, max_new, sample="greedy", seed=20260502, eos=-1):
        """The reference loop with a --sample spec and an rng seed (the head runs and
        the rng advances on every step, prompt steps included)."""
        mode, k, temp = parse_sample(sample)
        set_threads(self.threads)
        prompt = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(max(max_new, 1), np.int32)
        n = lib().b2o_generate_ex(C.byref(self.model), C.byref(self.state), _p(prompt, i32p),
                                  prompt.size, max_new, int(eos), mode, k, temp, seed & 0xFFFFFFFF,
                                  _p(out, i32p))
        if n < 0:
            raise OverflowError("KV cache overflow" if n == -1 else "bad token id")
        return out[:n].tolist()

    def generate(self, prompt, max_new):
        set_threads(self.threads)
        prompt = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(max(max_new, 1), np.int32)
        n = lib().b2o_generate(C.byref(self.model), C.byref(self.state), _p(prompt, i32p),
                               prompt.size, max_new, _p(out, i32p))
        if n < 0:
            raise OverflowError("KV cache overflow" if n == -1 else "bad token id")
        return out[:n].tolist()


def synth_tensors(plan, seed=0, stdv=0.02):
    """Host copy of a synthetic model (same generator as b2_create_synthetic)."""
    import importlib
    import sys
    root = str(HERE.parent)
    if root not in sys.path:
        sys.path.insert(0, root)
    pkg = importlib.import_module("aricode-ml_b200")
    from_name = pkg.runtime.fnv1a64
    out = {}
    for name, dt, shape, init in pkg.synth.tensor_specs(plan):
        tid = from_name(name)
        if dt == "i8":
            q, s = synth_quant(seed, tid, shape[0], shape[1], stdv)
            out[name] = q
            out[name + "_scales"] = s
        elif init == "rand":
            m, n = (shape if len(shape) == 2 else (1, shape[0]))
            a = synth_f32(seed, tid, m, n, stdv)
            out[name] = a if len(shape) == 2 else a[0]
        else:
            out[name] = np.full(shape, 1.0 if init == "ones" else 0.0, np.float32)
    return out
