"""Loader for the sm_100a C-ABI library ``libvbq.so`` (declared in include/vbq.h).

The library is built in-tree by ``vibeblade_b200/build.py``.  There is no fallback: if
the library is missing or fails to load, every operator raises.
"""
from __future__ import annotations

import ctypes as C
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libvbq.so"

VBQ_OK = 0
VBQ_ERR_TYPE = 1
VBQ_ERR_SHAPE = 2
VBQ_ERR_ALIGN = 3
VBQ_ERR_NULL = 4
VBQ_ERR_CUDA = 5
VBQ_ERR_TIMEOUT = 6
VBQ_ERR_UNSUPPORTED = 7
VBQ_ERR_WORKSPACE = 8

DTYPE_F32 = 0
DTYPE_BF16 = 1

# name -> (restype, argtypes); mirrors include/vbq.h
SIGNATURES = {
    "vbq_last_error": (C.c_char_p, []),
    "vbq_version": (C.c_int, []),
    "vbq_row_bytes": (C.c_int, [C.c_int32, C.c_int64, C.POINTER(C.c_int64)]),
    "vbq_dequantize": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_int32,
                                 C.c_int32, C.c_void_p]),
    "vbq_gemv_scratch_bytes": (C.c_int, [C.c_int64, C.c_int64, C.c_int32, C.c_int32,
                                         C.POINTER(C.c_size_t)]),
    "vbq_gemv": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_int32,
                           C.c_int32, C.c_void_p, C.c_size_t, C.c_void_p]),
    "vbq_device_status": (C.c_int, [C.POINTER(C.c_int32), C.c_int32]),
    "vbq_gemm_swiglu": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64,
                                  C.c_int64, C.c_int32, C.c_int64, C.c_void_p]),
    "vbq_gemm_ex": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_int64,
                              C.c_int32, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p]),
    "vbq_gemv_ex": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_int32,
                              C.c_int32, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t,
                              C.c_void_p]),
    "vbq_debug_wait_probe": (C.c_int, [C.c_int64, C.c_int32, C.c_void_p]),
    # data, flags (host arrays of device pointers), world, rank, epoch, n, out, timeout, stream
    "vbq_peer_allreduce": (C.c_int, [C.POINTER(C.c_void_p), C.POINTER(C.c_void_p), C.c_int32, C.c_int32,
                                     C.c_int32, C.c_int64, C.c_void_p, C.c_int64, C.c_void_p]),
    "vbq_ipc_export": (C.c_int, [C.c_void_p, C.c_void_p, C.POINTER(C.c_int64)]),
    "vbq_ipc_import": (C.c_int, [C.c_void_p, C.c_int64, C.POINTER(C.c_void_p)]),
    "vbq_ipc_close": (C.c_int, [C.c_void_p, C.c_int64]),
    "vbq_gemm": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_int64,
                           C.c_int32, C.c_int32, C.c_void_p]),
    "vbq_gemv_static_scratch": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64,
                                          C.c_int64, C.c_int32, C.c_int32, C.c_void_p]),
    "vbq_gemm_grouped": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p, C.c_int64,
                                   C.c_int64, C.c_int64, C.c_int32, C.c_int32, C.c_void_p,
                                   C.c_int32, C.c_void_p]),
    "vbq_moe_sort": (C.c_int, [C.c_void_p, C.c_int64, C.c_int32, C.c_int32, C.c_void_p,
                               C.c_void_p, C.c_void_p, C.c_void_p]),
    "vbq_moe_route": (C.c_int, [C.c_void_p, C.c_int64, C.c_int32, C.c_int32, C.c_void_p,
                                C.c_void_p, C.c_void_p]),
    "vbq_moe_workspace_bytes": (C.c_int, [C.c_int64, C.c_int64, C.c_int64, C.c_int32,
                                          C.c_int32, C.POINTER(C.c_size_t)]),
    "vbq_swiglu": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int32,
                             C.c_void_p]),
    "vbq_swiglu_rows": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_int32,
                                  C.c_void_p]),
    "vbq_moe_ffn": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                              C.c_void_p, C.c_int64, C.c_int64, C.c_int64, C.c_int32, C.c_int32,
                              C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_size_t,
                              C.c_void_p]),
}

_lock = threading.Lock()
_lib: C.CDLL | None = None


class VbqError(RuntimeError):
    """A non-zero status from libvbq; ``code`` is the VBQ_ERR_* value."""

    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


def load(path: str | os.PathLike | None = None) -> C.CDLL:
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"libvbq.so not found at {p}: build it with `python -m vibeblade_b200.build` "
                "(the k-quant path has no CPU fallback)")
        lib = C.CDLL(str(p))
        for name, (res, args) in SIGNATURES.items():
            f = getattr(lib, name)
            f.restype = res
            f.argtypes = args
        if path is None:
            _lib = lib
        return lib


def check(rc: int, lib: C.CDLL | None = None) -> None:
    if rc != VBQ_OK:
        lib = lib or load()
        msg = lib.vbq_last_error().decode(errors="replace")
        raise VbqError(rc, msg or f"libvbq error {rc}")
