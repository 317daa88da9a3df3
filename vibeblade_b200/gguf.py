"""GGUF weight source: the reference engine's ``GGUFFile`` over libvbq's reader.

Mirrors ``vibeblade::GGUFFile`` (kevin046/VibeBlade cpp/include/gguf.h,
cpp/src/gguf.cpp:14-320): ``version()``, ``file_size()``, ``tensors()``,
``tensor_info(name)``, ``tensor_data(name)``, ``meta_string / meta_int / meta_float /
meta_bool`` with the reference's defaults, and the array accessors; malformed files raise
``RuntimeError`` with the reference's message.  The parse runs in libvbq.so
(csrc/vbq_gguf.cpp, declared in include/vbq_gguf.h) over a read-only memory map.

On top of the reader, ``upload`` puts a tensor -- or a block-aligned tensor-parallel shard
of it -- into device memory as the raw blocks the kernels read, which replaces the
reference's raw-block upload (cpp/src/cuda_kernels.cu:152-156).
"""
from __future__ import annotations

import ctypes as C
from typing import NamedTuple

import numpy as np
import torch

from . import _lib
from . import formats as F


class TensorInfo(NamedTuple):
    """``vibeblade::TensorInfo`` (cpp/include/gguf.h:20-27)."""
    name: str
    n_dims: int
    dims: tuple[int, int, int, int]
    type: int
    offset: int
    size: int


class _TInfo(C.Structure):
    _fields_ = [("name", C.c_char_p), ("n_dims", C.c_int32), ("dims", C.c_int64 * 4),
                ("type", C.c_int32), ("offset", C.c_uint64), ("size", C.c_uint64)]


_SIGS = {
    "vbq_gguf_last_error": (C.c_char_p, []),
    "vbq_gguf_open": (C.c_int, [C.c_char_p, C.POINTER(C.c_void_p)]),
    "vbq_gguf_close": (None, [C.c_void_p]),
    "vbq_gguf_version": (C.c_int, [C.c_void_p, C.POINTER(C.c_uint32)]),
    "vbq_gguf_file_size": (C.c_int, [C.c_void_p, C.POINTER(C.c_uint64)]),
    "vbq_gguf_data_offset": (C.c_int, [C.c_void_p, C.POINTER(C.c_uint64)]),
    "vbq_gguf_n_tensors": (C.c_int, [C.c_void_p, C.POINTER(C.c_int64)]),
    "vbq_gguf_tensor": (C.c_int, [C.c_void_p, C.c_int64, C.POINTER(_TInfo)]),
    "vbq_gguf_find": (C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_int64)]),
    "vbq_gguf_tensor_data": (C.c_int, [C.c_void_p, C.c_int64, C.POINTER(C.c_void_p)]),
    "vbq_gguf_meta_count": (C.c_int, [C.c_void_p, C.c_char_p, C.c_int32, C.POINTER(C.c_int64)]),
    "vbq_gguf_meta_int": (C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_int64)]),
    "vbq_gguf_meta_float": (C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_double)]),
    "vbq_gguf_meta_bool": (C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_int32)]),
    "vbq_gguf_meta_string": (C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_void_p), C.POINTER(C.c_int64)]),
    "vbq_gguf_meta_int_array": (C.c_int, [C.c_void_p, C.c_char_p, C.c_void_p, C.c_int64, C.POINTER(C.c_int64)]),
    "vbq_gguf_meta_float_array": (C.c_int, [C.c_void_p, C.c_char_p, C.c_void_p, C.c_int64, C.POINTER(C.c_int64)]),
    "vbq_gguf_meta_string_at": (C.c_int, [C.c_void_p, C.c_char_p, C.c_int64, C.POINTER(C.c_void_p),
                                          C.POINTER(C.c_int64)]),
    "vbq_gguf_upload": (C.c_int, [C.c_void_p, C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_int64,
                                  C.c_void_p, C.c_int64, C.c_void_p]),
}

# metadata kinds (include/vbq_gguf.h)
META_INT, META_FLOAT, META_BOOL, META_STRING = 1, 2, 3, 4
META_INT_ARRAY, META_FLOAT_ARRAY, META_STRING_ARRAY = 5, 6, 7


def _lib_g():
    lib = _lib.load()
    if not getattr(lib, "_gguf_sigs", False):
        for name, (res, args) in _SIGS.items():
            f = getattr(lib, name)
            f.restype = res
            f.argtypes = args
        lib._gguf_sigs = True
    return lib


def _check(rc: int, lib) -> None:
    if rc != _lib.VBQ_OK:
        raise RuntimeError(lib.vbq_gguf_last_error().decode(errors="replace"))


class GGUFFile:
    """A parsed GGUF file (``vibeblade::GGUFFile``).  Use as a context manager or call
    ``close()``; arrays returned by ``tensor_data`` keep the file open while they live."""

    def __init__(self, path: str):
        lib = _lib_g()
        h = C.c_void_p()
        _check(lib.vbq_gguf_open(str(path).encode(), C.byref(h)), lib)
        self._lib = lib
        self._h = h
        self.path = str(path)

    # -- lifetime --
    def close(self) -> None:
        if getattr(self, "_h", None) is not None and self._h.value:
            self._lib.vbq_gguf_close(self._h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def _handle(self):
        if self._h is None:
            raise RuntimeError("GGUF: file is closed")
        return self._h

    # -- file --
    def version(self) -> int:
        v = C.c_uint32()
        _check(self._lib.vbq_gguf_version(self._handle(), C.byref(v)), self._lib)
        return int(v.value)

    def file_size(self) -> int:
        v = C.c_uint64()
        _check(self._lib.vbq_gguf_file_size(self._handle(), C.byref(v)), self._lib)
        return int(v.value)

    def data_offset(self) -> int:
        v = C.c_uint64()
        _check(self._lib.vbq_gguf_data_offset(self._handle(), C.byref(v)), self._lib)
        return int(v.value)

    # -- tensors --
    def _info(self, i: int) -> TensorInfo:
        t = _TInfo()
        _check(self._lib.vbq_gguf_tensor(self._handle(), i, C.byref(t)), self._lib)
        return TensorInfo(t.name.decode(errors="surrogateescape"), int(t.n_dims), tuple(int(d) for d in t.dims),
                          int(t.type), int(t.offset), int(t.size))

    def tensors(self) -> list[TensorInfo]:
        n = C.c_int64()
        _check(self._lib.vbq_gguf_n_tensors(self._handle(), C.byref(n)), self._lib)
        return [self._info(i) for i in range(n.value)]

    def _index(self, name: str) -> int:
        i = C.c_int64()
        _check(self._lib.vbq_gguf_find(self._handle(), name.encode(errors="surrogateescape"), C.byref(i)),
               self._lib)
        return int(i.value)

    def tensor_info(self, name: str) -> TensorInfo | None:
        i = self._index(name)
        return None if i < 0 else self._info(i)

    def tensor_data(self, name: str) -> np.ndarray | None:
        """The tensor's bytes (uint8, read-only, no copy), or None for an unknown name;
        raises when they run past the end of the file (gguf.cpp:255-262)."""
        i = self._index(name)
        if i < 0:
            return None
        info = self._info(i)
        p = C.c_void_p()
        _check(self._lib.vbq_gguf_tensor_data(self._handle(), i, C.byref(p)), self._lib)
        if info.size == 0:
            return np.zeros(0, np.uint8)
        buf = (C.c_uint8 * info.size).from_address(p.value)
        buf._owner = self  # the mapping stays alive while the array does
        a = np.frombuffer(buf, dtype=np.uint8)
        a.flags.writeable = False
        return a

    def matrix_shape(self, name: str) -> tuple[int, int, int]:
        """(K, N, type) of a weight tensor read as K rows of N values (N = dims[0])."""
        info = self.tensor_info(name)
        if info is None:
            raise RuntimeError(f"GGUF: no tensor '{name}'")
        K = 1
        for d in info.dims[1:info.n_dims]:
            K *= d
        return K, info.dims[0], info.type

    # the types the reference's dequant_row binding sizes rows for (cpp/src/bindings.cpp:
    # 416-425), anything else raising "Unsupported type for dequant_row"
    _DEQUANT_ROW_TYPES = (F.GGML_TYPE_F32, F.GGML_TYPE_F16, F.GGML_TYPE_Q4_0, F.GGML_TYPE_Q5_0,
                          F.GGML_TYPE_Q8_0, F.GGML_TYPE_Q4_K, F.GGML_TYPE_Q5_K, F.GGML_TYPE_Q6_K)

    def dequant_row(self, tensor_name: str, row_idx: int = 0, n_elements: int = 0,
                    device=None) -> np.ndarray:
        """``VibeBladeFast.dequant_row(tensor_name, row_idx=0, n_elements=0)``
        (cpp/src/bindings.cpp:407-436): row `row_idx` of a tensor (rows of dims[0] values),
        dequantized on the device, as fp32 numpy.  n_elements <= 0 means the whole row; a
        larger count runs on into the following rows, as there.  The same errors as the
        reference: "Tensor not found: <name>", "Unsupported type for dequant_row" (it takes
        F32, F16, Q4_0, Q5_0, Q8_0, Q4_K, Q5_K, Q6_K).  Unlike the reference, which reads
        whatever lies there, a row or count reaching past the tensor's bytes raises.  Q8_0
        rows decode the GGUF block (fp16 scale), not the reference CPU reader's fp32 one."""
        info = self.tensor_info(tensor_name)
        if info is None:
            raise RuntimeError(f"Tensor not found: {tensor_name}")
        t = info.type
        if t not in self._DEQUANT_ROW_TYPES:
            raise RuntimeError("Unsupported type for dequant_row")
        ne0 = info.dims[0]
        rb = F.row_bytes(t, ne0)
        n = int(n_elements) if n_elements > 0 else int(ne0)
        start, nbytes = int(row_idx) * rb, F.tensor_nbytes(t, n)
        data = self.tensor_data(tensor_name)
        if row_idx < 0 or start + nbytes > data.size:
            raise RuntimeError(f"dequant_row: row {row_idx} x {n} values of '{tensor_name}' runs past "
                               f"its {data.size} bytes")
        from .dequant import dequantize_row
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        row = torch.from_numpy(np.array(data[start:start + nbytes])).to(dev)
        return dequantize_row(row, None, n, t).cpu().numpy()

    # -- metadata (the reference's defaults when a key is missing) --
    def meta_count(self, key: str, kind: int) -> int | None:
        """Length of `key`'s value of `kind` (META_*; 1 for a scalar), or None without one."""
        n = C.c_int64()
        rc = self._lib.vbq_gguf_meta_count(self._handle(), key.encode(), kind, C.byref(n))
        return int(n.value) if rc == _lib.VBQ_OK else None

    def meta_int(self, key: str, default: int = 0) -> int:
        v = C.c_int64()
        rc = self._lib.vbq_gguf_meta_int(self._handle(), key.encode(), C.byref(v))
        return int(v.value) if rc == _lib.VBQ_OK else default

    def meta_float(self, key: str, default: float = 0.0) -> float:
        v = C.c_double()
        rc = self._lib.vbq_gguf_meta_float(self._handle(), key.encode(), C.byref(v))
        return float(v.value) if rc == _lib.VBQ_OK else default

    def meta_bool(self, key: str, default: bool = False) -> bool:
        v = C.c_int32()
        rc = self._lib.vbq_gguf_meta_bool(self._handle(), key.encode(), C.byref(v))
        return bool(v.value) if rc == _lib.VBQ_OK else default

    def meta_string(self, key: str) -> str:
        p, n = C.c_void_p(), C.c_int64()
        rc = self._lib.vbq_gguf_meta_string(self._handle(), key.encode(), C.byref(p), C.byref(n))
        return C.string_at(p.value, n.value).decode(errors="surrogateescape") if rc == _lib.VBQ_OK and n.value else ""

    def meta_int_array(self, key: str) -> list[int]:
        n = C.c_int64()
        if self._lib.vbq_gguf_meta_int_array(self._handle(), key.encode(), None, 0, C.byref(n)) != _lib.VBQ_OK:
            return []
        out = (C.c_int64 * max(n.value, 1))()
        self._lib.vbq_gguf_meta_int_array(self._handle(), key.encode(), out, n.value, C.byref(n))
        return [int(v) for v in out[:n.value]]

    def meta_float_array(self, key: str) -> list[float]:
        n = C.c_int64()
        if self._lib.vbq_gguf_meta_float_array(self._handle(), key.encode(), None, 0, C.byref(n)) != _lib.VBQ_OK:
            return []
        out = (C.c_float * max(n.value, 1))()
        self._lib.vbq_gguf_meta_float_array(self._handle(), key.encode(), out, n.value, C.byref(n))
        return [float(v) for v in out[:n.value]]

    def meta_string_array(self, key: str) -> list[str]:
        n = self.meta_count(key, META_STRING_ARRAY)
        if n is None:
            return []
        res = []
        p, ln = C.c_void_p(), C.c_int64()
        for j in range(n):
            _check(self._lib.vbq_gguf_meta_string_at(self._handle(), key.encode(), j, C.byref(p), C.byref(ln)),
                   self._lib)
            res.append(C.string_at(p.value, ln.value).decode(errors="surrogateescape") if ln.value else "")
        return res

    # -- device upload --
    def upload(self, name: str, device, rows: tuple[int, int] | None = None,
               cols: tuple[int, int] | None = None, row_bytes: int | None = None) -> torch.Tensor:
        """Rows [r0, r1) x columns [c0, c1) (whole blocks) of tensor `name` as a uint8
        device tensor [r1 - r0, row_bytes] of raw blocks (row_bytes defaults to the shard's
        own; larger values pad each row with zeros).  Runs on the device's current stream
        and returns when the copy is done."""
        i = self._index(name)
        if i < 0:
            raise RuntimeError(f"GGUF: no tensor '{name}'")
        K, N, t = self.matrix_shape(name)
        r0, r1 = rows if rows is not None else (0, K)
        c0, c1 = cols if cols is not None else (0, N)
        bv = F.BLOCK_VALUES.get(t)
        if bv is None:
            raise RuntimeError(f"GGUF: tensor '{name}' has type {t}, which this library does not read")
        wb = (c1 - c0) // bv * F.BLOCK_BYTES[t]
        rb = wb if row_bytes is None else int(row_bytes)
        dev = torch.device(device)
        out = torch.empty((r1 - r0, rb), dtype=torch.uint8, device=dev)
        with torch.cuda.device(dev):
            sp = torch.cuda.current_stream(dev).cuda_stream
            _check(self._lib.vbq_gguf_upload(self._handle(), i, r0, r1, c0, c1, out.data_ptr(), rb, sp),
                   self._lib)
        return out

    def upload_shard(self, name: str, kind: str, rank: int, world: int, device) -> torch.Tensor:
        """Rank `rank`'s tensor-parallel shard of weight `name`, read straight from the
        file: a column split takes output columns [r N / W, (r + 1) N / W) of every row, a
        row split input rows [r K / W, (r + 1) K / W) -- the same bytes as
        ``vibeblade_b200.tp.shard`` of the whole tensor, without uploading the rest."""
        from .tp import check_split
        K, N, t = self.matrix_shape(name)
        check_split(kind, K, N, t, world)
        if kind == "column":
            n = N // world
            return self.upload(name, device, cols=(rank * n, (rank + 1) * n))
        k = K // world
        return self.upload(name, device, rows=(rank * k, (rank + 1) * k))
