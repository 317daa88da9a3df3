"""ctypes faces of the two CPU checkers (TEST INFRASTRUCTURE ONLY).

``Oracle`` wraps the C restatement (oracle/vbq_oracle.c).  ``RefLib`` wraps the
reference's own ``vibeblade::dequantize_row`` / ``gemv_dequant`` / ``gemv_dequant_mt``
compiled from its sources (cpp/include/dequant.h:11-48) by oracle/build.py.
"""
from __future__ import annotations

import ctypes as C
import os
from concurrent.futures import ThreadPoolExecutor
from functools import lru_cache

import numpy as np

from . import build as _build

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")

BLOCK_VALUES = {0: 1, 1: 1, 30: 1, 2: 32, 3: 32, 6: 32, 7: 32, 8: 32,
                10: 256, 11: 256, 12: 256, 13: 256, 14: 256, 15: 256}
BLOCK_BYTES = {0: 4, 1: 2, 30: 2, 2: 18, 3: 20, 6: 22, 7: 24, 8: 34,
               10: 84, 11: 110, 12: 144, 13: 176, 14: 210, 15: 292}


def row_bytes(qtype: int, n: int) -> int:
    return (n // BLOCK_VALUES[qtype]) * BLOCK_BYTES[qtype]


def _u8(w) -> np.ndarray:
    a = np.ascontiguousarray(w)
    return a.view(np.uint8).reshape(-1)


class Oracle:
    """The C restatement.  All functions return numpy arrays."""

    def __init__(self, path: str):
        lib = C.CDLL(path)
        self.lib = lib
        lib.vbo_f16_to_f32.argtypes = [C.c_uint16]
        lib.vbo_f16_to_f32.restype = C.c_float
        lib.vbo_f16_to_f32_ieee.argtypes = [C.c_uint16]
        lib.vbo_f16_to_f32_ieee.restype = C.c_float
        for name in ("vbo_dequantize_row_q4_K", "vbo_dequantize_row_q6_K",
                     "vbo_dequantize_row_q8_0", "vbo_dequantize_row_q8_0_f32scale"):
            f = getattr(lib, name)
            f.argtypes = [_u8p, _f32p, C.c_int64]
            f.restype = None
        lib.vbo_dequantize_row.argtypes = [_u8p, _f32p, C.c_int64, C.c_int32]
        lib.vbo_dequantize_row.restype = C.c_int
        lib.vbo_dequantize_matrix.argtypes = [_u8p, _f32p, C.c_int64, C.c_int64, C.c_int32]
        lib.vbo_dequantize_matrix.restype = C.c_int
        lib.vbo_gemv_dequant_batch.argtypes = [_f32p, _u8p, _f32p, C.c_int64, C.c_int64,
                                               C.c_int32, C.c_int64]
        lib.vbo_gemv_dequant_batch.restype = C.c_int
        lib.vbo_gemm_f64.argtypes = [_f32p, _u8p, _f64p, C.c_int64, C.c_int64, C.c_int64,
                                     C.c_int32]
        lib.vbo_gemm_f64.restype = C.c_int
        lib.vbo_row_bytes.argtypes = [C.c_int32, C.c_int64]
        lib.vbo_row_bytes.restype = C.c_int64

    def f16_to_f32(self, h: int) -> float:
        """The reference's conversion (doubles subnormals)."""
        return self.lib.vbo_f16_to_f32(h)

    def f16_to_f32_ieee(self, h: int) -> float:
        return self.lib.vbo_f16_to_f32_ieee(h)

    def dequantize_row(self, row, n: int, qtype: int) -> np.ndarray:
        out = np.zeros(n, np.float32)
        if self.lib.vbo_dequantize_row(_u8(row), out, n, qtype) != 0:
            raise RuntimeError(f"Unsupported dequant type: {qtype}")
        return out

    def dequantize_q8_0_f32scale(self, row, n: int) -> np.ndarray:
        out = np.zeros(n, np.float32)
        self.lib.vbo_dequantize_row_q8_0_f32scale(_u8(row), out, n)
        return out

    def dequantize(self, w, K: int, N: int, qtype: int) -> np.ndarray:
        out = np.zeros((K, N), np.float32)
        if self.lib.vbo_dequantize_matrix(_u8(w), out.reshape(-1), K, N, qtype) != 0:
            raise RuntimeError(f"Unsupported dequant type: {qtype}")
        return out

    def gemv_dequant(self, x, w, K: int, N: int, qtype: int) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        batch = x.size // K
        out = np.zeros((batch, N), np.float32)
        rc = self.lib.vbo_gemv_dequant_batch(x.reshape(-1), _u8(w), out.reshape(-1), K, N,
                                            qtype, batch)
        if rc != 0:
            raise RuntimeError(f"gemv_dequant: unsupported type {qtype}")
        return out

    def gemm_f64(self, a_f32, w, M: int, K: int, N: int, qtype: int) -> np.ndarray:
        a = np.ascontiguousarray(a_f32, np.float32).reshape(-1)
        out = np.zeros((M, N), np.float64)
        if self.lib.vbo_gemm_f64(a, _u8(w), out.reshape(-1), M, K, N, qtype) != 0:
            raise RuntimeError(f"gemm: unsupported type {qtype}")
        return out


class RefLib:
    """The reference's own CPU functions, called through their C++ symbols."""

    _SYM = {
        "dequantize_row": "_ZN9vibeblade14dequantize_rowEPKvPflNS_9ggml_typeE",
        "gemv_dequant": "_ZN9vibeblade12gemv_dequantEPKfPKvPfllNS_9ggml_typeES4_",
        "gemv_dequant_mt": "_ZN9vibeblade15gemv_dequant_mtEPKfPKvPfllNS_9ggml_typeEiS4_",
    }

    def __init__(self, path: str):
        lib = C.CDLL(path)
        self.lib = lib
        self.path = path
        self._deq = getattr(lib, self._SYM["dequantize_row"])
        self._deq.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_int32]
        self._deq.restype = None
        self._gemv = getattr(lib, self._SYM["gemv_dequant"])
        self._gemv.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64,
                               C.c_int32, C.c_void_p]
        self._gemv.restype = None
        self._gemv_mt = getattr(lib, self._SYM["gemv_dequant_mt"])
        self._gemv_mt.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64,
                                  C.c_int32, C.c_int, C.c_void_p]
        self._gemv_mt.restype = None

    def dequantize_row(self, row, n: int, qtype: int) -> np.ndarray:
        # The reference's C++ Q8_0 reader takes quants from bytes 4..35 of each 34-byte
        # block, i.e. 2 bytes past the row's end on the last block: read from a padded copy.
        src = _u8(row)
        r = np.zeros(src.size + 64, np.uint8)
        r[:src.size] = src
        # The reference's Q4_K loop writes whole 64-value groups even for a ragged tail
        # (cpp/src/dequant.cpp:282-296), so give it room for a full block.
        out = np.zeros(((n + 255) // 256) * 256, np.float32)
        self._deq(r.ctypes.data, out.ctypes.data, n, qtype)
        return out[:n].copy()

    def gemv_dequant(self, x, w, K: int, N: int, qtype: int) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        batch = x.size // K
        xs = x.reshape(batch, K)
        wb = _u8(w)
        out = np.zeros((batch, N), np.float32)
        scratch = np.zeros(N, np.float32)
        for b in range(batch):
            self._gemv(xs[b].ctypes.data, wb.ctypes.data, out[b].ctypes.data, K, N, qtype,
                       scratch.ctypes.data)
        return out

    def gemv_dequant_sliced(self, x, w, K: int, N: int, qtype: int, threads: int,
                            pool: ThreadPoolExecutor | None = None) -> np.ndarray:
        """Timing harness: the reference's gemv_dequant run on `threads` disjoint K
        slices at once (ctypes releases the GIL), partial outputs summed after.  The
        reference's own gemv_dequant_mt ignores n_threads (cpp/src/dequant.cpp:783-792);
        this only lets the timed CPU baseline use the host's cores."""
        x = np.ascontiguousarray(x, np.float32)
        batch = x.size // K
        xs = x.reshape(batch, K)
        wb = _u8(w)
        rb = row_bytes(qtype, N)
        threads = max(1, min(threads, K))
        bounds = np.linspace(0, K, threads + 1).astype(np.int64)
        parts = np.zeros((threads, batch, N), np.float32)
        scratch = np.zeros((threads, N), np.float32)

        def run(t):
            k0, k1 = int(bounds[t]), int(bounds[t + 1])
            if k1 <= k0:
                return
            for b in range(batch):
                self._gemv(xs[b, k0:].ctypes.data, wb.ctypes.data + k0 * rb,
                           parts[t, b].ctypes.data, k1 - k0, N, qtype,
                           scratch[t].ctypes.data)

        if threads == 1:
            run(0)
        else:
            own = pool is None
            ex = pool or ThreadPoolExecutor(threads)
            list(ex.map(run, range(threads)))
            if own:
                ex.shutdown()
        return parts.sum(axis=0, dtype=np.float32)


@lru_cache(maxsize=1)
def load_oracle() -> Oracle:
    return Oracle(str(_build.build_oracle()))


@lru_cache(maxsize=1)
def load_ref_avx2() -> RefLib | None:
    """The reference built with its AVX2 release flags (timing only), when the library
    exists and this host's CPU has AVX2 and FMA; else None."""
    if load_ref() is None or not _build.host_has_avx2():
        return None
    p = _build.REF_AVX2_SO
    return RefLib(str(p)) if p.exists() else None


@lru_cache(maxsize=1)
def load_ref() -> RefLib | None:
    """The compiled reference, or None when neither its sources nor a prebuilt copy
    exist."""
    p = _build.build_ref() if os.environ.get("VB_NO_REF_BUILD") is None else (
        _build.REF_SO if _build.REF_SO.exists() else None)
    return RefLib(str(p)) if p is not None and os.path.exists(p) else None


class RefGGUF:
    """The reference's own GGUF reader (vibeblade::GGUFFile) through oracle/ref_gguf_shim.cpp."""

    def __init__(self, path: str):
        lib = C.CDLL(path)
        self.lib = lib
        sig = {
            "vbr_gguf_error": (C.c_char_p, []),
            "vbr_gguf_open": (C.c_void_p, [C.c_char_p]),
            "vbr_gguf_close": (None, [C.c_void_p]),
            "vbr_gguf_version": (C.c_int64, [C.c_void_p]),
            "vbr_gguf_n_tensors": (C.c_int64, [C.c_void_p]),
            "vbr_gguf_tensor": (C.c_int, [C.c_void_p, C.c_int64, C.c_char_p, C.c_int64, C.POINTER(C.c_int32),
                                          C.POINTER(C.c_int64), C.POINTER(C.c_int32), C.POINTER(C.c_uint64),
                                          C.POINTER(C.c_uint64)]),
            "vbr_gguf_tensor_data": (C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_void_p)]),
            "vbr_gguf_has_tensor": (C.c_int, [C.c_void_p, C.c_char_p]),
            "vbr_gguf_meta_int": (C.c_int64, [C.c_void_p, C.c_char_p, C.c_int64]),
            "vbr_gguf_meta_float": (C.c_double, [C.c_void_p, C.c_char_p, C.c_double]),
            "vbr_gguf_meta_bool": (C.c_int, [C.c_void_p, C.c_char_p, C.c_int]),
            "vbr_gguf_meta_string": (C.c_int64, [C.c_void_p, C.c_char_p, C.c_char_p, C.c_int64]),
            "vbr_gguf_meta_int_array": (C.c_int64, [C.c_void_p, C.c_char_p, C.POINTER(C.c_int64), C.c_int64]),
            "vbr_gguf_meta_float_array": (C.c_int64, [C.c_void_p, C.c_char_p, C.POINTER(C.c_float), C.c_int64]),
            "vbr_gguf_meta_string_array_len": (C.c_int64, [C.c_void_p, C.c_char_p]),
            "vbr_gguf_meta_string_at": (C.c_int64, [C.c_void_p, C.c_char_p, C.c_int64, C.c_char_p, C.c_int64]),
        }
        for name, (res, args) in sig.items():
            f = getattr(lib, name)
            f.restype, f.argtypes = res, args

    def open(self, path: str):
        """(handle, None) or (None, the reference's exception message)."""
        h = self.lib.vbr_gguf_open(str(path).encode())
        return (h, None) if h else (None, self.lib.vbr_gguf_error().decode())

    def close(self, h) -> None:
        self.lib.vbr_gguf_close(h)

    def tensors(self, h) -> list[tuple]:
        out = []
        buf = C.create_string_buffer(4096)
        for i in range(self.lib.vbr_gguf_n_tensors(h)):
            nd, ty = C.c_int32(), C.c_int32()
            dims = (C.c_int64 * 4)()
            off, size = C.c_uint64(), C.c_uint64()
            self.lib.vbr_gguf_tensor(h, i, buf, 4096, C.byref(nd), dims, C.byref(ty), C.byref(off), C.byref(size))
            out.append((buf.value.decode(errors="surrogateescape"), nd.value, tuple(dims), ty.value, off.value,
                        size.value))
        return out

    def tensor_data(self, h, name: str, size: int):
        """bytes, None when absent, or the exception message (str) when it throws"""
        p = C.c_void_p()
        rc = self.lib.vbr_gguf_tensor_data(h, name.encode(), C.byref(p))
        if rc < 0:
            return self.lib.vbr_gguf_error().decode()
        return None if rc == 0 else C.string_at(p.value, size)

    def meta_string(self, h, key):
        n = self.lib.vbr_gguf_meta_string(h, key.encode(), None, 0)
        buf = C.create_string_buffer(n + 1)
        self.lib.vbr_gguf_meta_string(h, key.encode(), buf, n + 1)
        return buf.raw[:n].decode(errors="surrogateescape")

    def meta_int_array(self, h, key):
        n = self.lib.vbr_gguf_meta_int_array(h, key.encode(), None, 0)
        a = (C.c_int64 * max(n, 1))()
        self.lib.vbr_gguf_meta_int_array(h, key.encode(), a, n)
        return [int(v) for v in a[:n]]

    def meta_float_array(self, h, key):
        n = self.lib.vbr_gguf_meta_float_array(h, key.encode(), None, 0)
        a = (C.c_float * max(n, 1))()
        self.lib.vbr_gguf_meta_float_array(h, key.encode(), a, n)
        return [float(v) for v in a[:n]]

    def meta_string_array(self, h, key):
        res = []
        for j in range(self.lib.vbr_gguf_meta_string_array_len(h, key.encode())):
            n = self.lib.vbr_gguf_meta_string_at(h, key.encode(), j, None, 0)
            buf = C.create_string_buffer(n + 1)
            self.lib.vbr_gguf_meta_string_at(h, key.encode(), j, buf, n + 1)
            res.append(buf.raw[:n].decode(errors="surrogateescape"))
        return res


@lru_cache(maxsize=1)
def load_ref_gguf() -> RefGGUF | None:
    """The reference's GGUF reader, or None when it cannot be built or found."""
    p = _build.build_ref_gguf() if os.environ.get("VB_NO_REF_BUILD") is None else (
        _build.REF_GGUF_SO if _build.REF_GGUF_SO.exists() else None)
    return RefGGUF(str(p)) if p is not None and os.path.exists(p) else None
