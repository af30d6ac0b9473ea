"""The ``--target b200`` weight blob: one file, tensors ready for a single H2D copy.

Layout (little-endian):

====== ======== ==========================================================
offset size     field
====== ======== ==========================================================
0      8        magic ``B2DBLOB1``
8      4        version (1)
12     4        number of tensors
16     8        offset of the tensor table (always 64)
24     8        offset of the data region (4096-aligned)
32     8        bytes in the data region
40     8        checksum of the data region (see :func:`checksum`)
48     4        bytes of the embedded plan JSON
52     4        reserved
56     8        offset of the embedded plan JSON
64     128*n    tensor table
====== ======== ==========================================================

Each 128-byte table entry: name (64 bytes, NUL padded), dtype u32 (1 = int8,
2 = f32, 3 = int4: two codes per byte, the even column in the low nibble, as the
reference's ``.i4`` files), ndim u32, shape u64[2] (int4: the logical columns),
ld u64 (row stride in elements; int4: in bytes), offset u64 (relative to the
data region, 256-aligned), nbytes u64, 16 reserved bytes.

2-D int8 tensors keep the reference's row-major codes with each row padded with
zero bytes to a multiple of 16 (so every row starts on a 16-byte boundary for
the TMA bulk copies); 2-D f32 tensors pad rows to a multiple of 4 elements.
Codes and scales are byte-identical to the reference's ``.i8`` /
``_scales.f32`` staging files row by row (aricode_pack.py:3356-3379).
"""
from __future__ import annotations

import json
import struct
from dataclasses import dataclass

import numpy as np

MAGIC = b"B2DBLOB1"
VERSION = 1
DT_I8, DT_F32, DT_I4 = 1, 2, 3
_HDR = struct.Struct("<8sIIQQQQIIQ")
_ENT = struct.Struct("<64sII2QQQQ16x")
assert _HDR.size == 64 and _ENT.size == 128

_MIX1 = np.uint64(0x9E3779B97F4A7C15)
_MIX2 = np.uint64(0xBF58476D1CE4E5B9)


def row_stride(cols, dtype_code):
    """Padded row stride in elements for a 2-D tensor."""
    if dtype_code in (DT_I8, DT_I4):
        return (cols + 15) // 16 * 16
    return (cols + 3) // 4 * 4


def checksum(buf: np.ndarray) -> int:
    """sum_i ((w_i xor i*0x9E3779B97F4A7C15) * 0xBF58476D1CE4E5B9) mod 2^64 over the
    data region read as little-endian u64 words (zero-padded to 8 bytes). The same
    loop runs in the C++ loader."""
    b = np.ascontiguousarray(buf).view(np.uint8).ravel()
    pad = (-b.size) % 8
    if pad:
        b = np.concatenate([b, np.zeros(pad, np.uint8)])
    w = b.view("<u8")
    total = np.uint64(0)
    chunk = 1 << 24
    with np.errstate(over="ignore"):
        for s in range(0, w.size, chunk):
            idx = np.arange(s, min(s + chunk, w.size), dtype=np.uint64)
            total = total + np.sum((w[s:s + chunk] ^ (idx * _MIX1)) * _MIX2, dtype=np.uint64)
    return int(total)


@dataclass
class TensorEntry:
    name: str
    dtype: int
    shape: tuple
    ld: int
    offset: int
    nbytes: int


def write_blob(path, tensors: dict, plan: dict):
    """tensors: name -> np.ndarray (int8 or float32, 1-D or 2-D, unpadded)."""
    entries, chunks = [], []
    off = 0
    for name, arr in tensors.items():
        arr = np.asarray(arr)
        if arr.dtype == np.int8:
            code = DT_I8
        elif arr.dtype == np.uint8:
            code = DT_I4                    # packed nibbles [rows, cols / 2]
        elif arr.dtype == np.float32:
            code = DT_F32
        else:
            raise TypeError(f"{name}: unsupported dtype {arr.dtype}")
        if len(name.encode()) >= 64:
            raise ValueError(f"tensor name too long: {name}")
        if arr.ndim == 1:
            shape, ld, data = (arr.shape[0], 1), arr.shape[0], arr
        elif arr.ndim == 2:
            rows, cols = arr.shape
            ld = row_stride(cols, code)
            data = np.zeros((rows, ld), arr.dtype)
            data[:, :cols] = arr
            shape = (rows, 2 * cols if code == DT_I4 else cols)
        else:
            raise ValueError(f"{name}: only 1-D/2-D tensors")
        raw = np.ascontiguousarray(data).view(np.uint8).ravel()
        off = (off + 255) // 256 * 256
        entries.append(TensorEntry(name, code, shape if arr.ndim == 2 else (arr.shape[0],),
                                   ld, off, raw.size))
        chunks.append((off, raw))
        off += raw.size
    data_bytes = (off + 255) // 256 * 256
    data = np.zeros(data_bytes, np.uint8)
    for o, raw in chunks:
        data[o:o + raw.size] = raw
    plan_raw = json.dumps(plan, indent=1, sort_keys=True).encode()
    table_off = 64
    plan_off = table_off + 128 * len(entries)
    data_off = (plan_off + len(plan_raw) + 4095) // 4096 * 4096
    hdr = _HDR.pack(MAGIC, VERSION, len(entries), table_off, data_off, data_bytes,
                    checksum(data), len(plan_raw), 0, plan_off)
    with open(path, "wb") as f:
        f.write(hdr)
        for e in entries:
            ndim = len(e.shape)
            shp = (e.shape[0], e.shape[1] if ndim == 2 else 0)
            f.write(_ENT.pack(e.name.encode(), e.dtype, ndim, shp[0], shp[1], e.ld,
                              e.offset, e.nbytes))
        f.write(plan_raw)
        f.write(b"\0" * (data_off - plan_off - len(plan_raw)))
        f.write(data.tobytes())
    return entries


def read_blob(path, verify=True):
    """Returns (plan, {name: np.ndarray}) with 2-D tensors cut back to their
    logical width (views onto the padded data)."""
    with open(path, "rb") as f:
        raw = f.read()
    magic, ver, n, table_off, data_off, data_bytes, csum, plan_len, _, plan_off = \
        _HDR.unpack_from(raw, 0)
    if magic != MAGIC or ver != VERSION:
        raise ValueError(f"{path}: not a b200 decode blob (magic {magic!r}, version {ver})")
    data = np.frombuffer(raw, np.uint8, data_bytes, data_off)
    if verify and checksum(data) != csum:
        raise ValueError(f"{path}: checksum mismatch")
    plan = json.loads(raw[plan_off:plan_off + plan_len].decode())
    out = {}
    for i in range(n):
        name, code, ndim, s0, s1, ld, off, nbytes = _ENT.unpack_from(raw, table_off + 128 * i)
        name = name.rstrip(b"\0").decode()
        dt = {DT_I8: np.int8, DT_I4: np.uint8}.get(code, np.float32)
        arr = np.frombuffer(data, dt, nbytes // np.dtype(dt).itemsize, off)
        if ndim == 2:
            arr = arr.reshape(s0, ld)[:, :(s1 // 2 if code == DT_I4 else s1)]
        out[name] = arr
    return plan, out
