"""Write GGUF v3 files for the tests (test helper, not product code).

The layout is the GGUF container the reference reads (cpp/src/gguf.cpp:62-193) and the
reference's own test helper writes (tests/test_loader.py:35-118): header (magic, version,
tensor count, kv count), key/value pairs, tensor infos, the data section at the next
multiple of 32 bytes.  Values are given with their GGUF type id so every kind can be
written, and field overrides let tests build malformed files.
"""
from __future__ import annotations

import struct

import numpy as np

MAGIC = 0x46554747

# GGUF metadata value type ids
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f",
           BOOL: "<?", U64: "<Q", I64: "<q", F64: "<d"}


def enc_str(s) -> bytes:
    b = s.encode() if isinstance(s, str) else bytes(s)
    return struct.pack("<Q", len(b)) + b


def _value(vtype: int, value) -> bytes:
    if vtype == STRING:
        return enc_str(value)
    if vtype == ARRAY:
        etype, items = value
        out = struct.pack("<IQ", etype, len(items))
        for it in items:
            out += _value(etype, it)
        return out
    return struct.pack(_SCALAR[vtype], value)


def build(kv: list[tuple[str, int, object]], tensors: list[tuple[str, tuple[int, ...], int, bytes]],
          version: int = 3, magic: int = MAGIC, n_tensors: int | None = None, n_kv: int | None = None,
          align: int = 32, offsets: list[int] | None = None) -> bytes:
    """kv: (key, value type id, value); an ARRAY value is (element type id, [items]).
    tensors: (name, dims with dims[0] the fastest, ggml type id, data bytes).  Tensor data
    is placed back to back, each at a multiple of `align`, unless `offsets` gives them."""
    out = struct.pack("<IIQQ", magic, version, len(tensors) if n_tensors is None else n_tensors,
                      len(kv) if n_kv is None else n_kv)
    for key, vt, val in kv:
        out += enc_str(key) + struct.pack("<I", vt) + _value(vt, val)
    offs, pos = [], 0
    for i, (_, _, _, data) in enumerate(tensors):
        o = offsets[i] if offsets is not None else pos
        offs.append(o)
        pos = o + len(data)
        pos = (pos + align - 1) // align * align
    for (name, dims, ttype, _), o in zip(tensors, offs):
        out += enc_str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        out += struct.pack("<IQ", ttype, o)
    data_start = (len(out) + 31) // 32 * 32
    out += b"\0" * (data_start - len(out))
    body = bytearray(max([o + len(t[3]) for o, t in zip(offs, tensors)], default=0))
    for (_, _, _, data), o in zip(tensors, offs):
        body[o:o + len(data)] = data
    return out + bytes(body)


def write(path, *args, **kw) -> str:
    with open(path, "wb") as f:
        f.write(build(*args, **kw))
    return str(path)


def weight_tensor(name: str, w_bytes, K: int, N: int, ttype: int):
    """A K x N weight (rows of blocks, the layout gemv_dequant reads) as a GGUF tensor:
    dims (N, K)."""
    data = w_bytes if isinstance(w_bytes, (bytes, bytearray)) else np.ascontiguousarray(w_bytes).tobytes()
    return (name, (N, K), ttype, bytes(data))
