"""The C-ABI library: builds for sm_100a, loads, and exports every function include/*.h
declares.  Only host-side argument checks run here (no GPU in this container)."""
from __future__ import annotations

import ctypes as C
import re
import subprocess

import pytest

from conftest import ROOT


def declared_functions() -> set[str]:
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(vbq_\w+)\s*\(", text, re.M):
            names.add(m.group(1))
    return names


@pytest.fixture(scope="module")
def lib():
    from vibeblade_b200 import _lib
    return _lib.load()


def test_header_declares_entry_points():
    names = declared_functions()
    assert {"vbq_dequantize", "vbq_gemv", "vbq_last_error", "vbq_row_bytes"} <= names


def test_library_exports_every_declared_symbol(lib):
    from vibeblade_b200 import _lib
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    missing = declared_functions() - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"
    for name in declared_functions():
        getattr(lib, name)  # resolvable through the dynamic loader


def test_row_bytes(lib):
    v = C.c_int64()
    assert lib.vbq_row_bytes(12, 4096, C.byref(v)) == 0 and v.value == 16 * 144
    assert lib.vbq_row_bytes(14, 4096, C.byref(v)) == 0 and v.value == 16 * 210
    assert lib.vbq_row_bytes(8, 4096, C.byref(v)) == 0 and v.value == 128 * 34
    # the reference dispatcher's other block types (cpp/src/dequant.cpp:753-763)
    for t, bv, bb in ((2, 32, 18), (3, 32, 20), (6, 32, 22), (7, 32, 24), (10, 256, 84),
                      (11, 256, 110), (13, 256, 176), (15, 256, 292)):
        assert lib.vbq_row_bytes(t, 4096, C.byref(v)) == 0 and v.value == 4096 // bv * bb, t
    # Q8_1 (9) and unknown ids: the reference throws (cpp/src/dequant.cpp:423)
    assert lib.vbq_row_bytes(9, 4096, C.byref(v)) == 1
    assert b"Unsupported dequant type: 9" in lib.vbq_last_error()
    assert lib.vbq_row_bytes(4, 4096, C.byref(v)) == 1


def test_argument_errors_need_no_gpu(lib):
    from vibeblade_b200 import _lib
    # unsupported type: reference message (cpp/src/dequant.cpp:764)
    assert lib.vbq_gemv(None, None, None, 16, 256, 9, 1, None, 0, None) == _lib.VBQ_ERR_TYPE
    assert lib.vbq_last_error() == b"gemv_dequant: unsupported type 9"
    assert lib.vbq_gemv(None, None, None, 16, 256, 12, 33, None, 0, None) == _lib.VBQ_ERR_SHAPE
    assert lib.vbq_gemv(None, None, None, 16, 300, 12, 1, None, 0, None) == _lib.VBQ_ERR_SHAPE
    assert lib.vbq_gemv(None, None, None, 16, 256, 12, 1, None, 0, None) == _lib.VBQ_ERR_NULL
    assert lib.vbq_gemv(16, 16, 8, 16, 256, 12, 1, None, 0, None) == _lib.VBQ_ERR_ALIGN
    assert lib.vbq_dequantize(None, None, 2, 100, 12, 0, None) == _lib.VBQ_ERR_SHAPE
    assert lib.vbq_dequantize(None, None, 1, 256, 9, 0, None) == _lib.VBQ_ERR_TYPE
    assert lib.vbq_dequantize(None, None, 2, 100, 2, 0, None) == _lib.VBQ_ERR_SHAPE  # Q4_0: 32s
    assert lib.vbq_gemv(None, None, None, 16, 100, 13, 1, None, 0, None) == _lib.VBQ_ERR_SHAPE
    assert lib.vbq_gemv(None, None, None, 16, 96, 6, 1, None, 0, None) == _lib.VBQ_ERR_NULL  # Q5_0 N=96 ok
    # the other block types take the generic kernel: no scratch, any batch
    v = C.c_size_t(7)
    assert lib.vbq_gemv_scratch_bytes(4096, 14336, 13, 100, C.byref(v)) == 0 and v.value == 0
    assert lib.vbq_gemm(None, None, None, 64, 256, 256, 13, 0, None) == _lib.VBQ_ERR_TYPE
    assert lib.vbq_dequantize(None, None, 1, 256, 12, 5, None) == _lib.VBQ_ERR_SHAPE
    assert lib.vbq_dequantize(0, 0, 0, 256, 12, 0, None) == _lib.VBQ_OK  # empty: no work


def test_newer_entry_points_validate_before_any_cuda_call(lib):
    """vbq_swiglu_rows and vbq_moe_sort check their arguments before touching the GPU."""
    from vibeblade_b200 import _lib
    assert lib.vbq_swiglu_rows(None, None, 4, 16, 9, None) == _lib.VBQ_ERR_SHAPE      # dtype
    assert lib.vbq_swiglu_rows(None, None, -1, 16, 0, None) == _lib.VBQ_ERR_SHAPE     # rows < 0
    assert lib.vbq_swiglu_rows(None, None, 0, 16, 0, None) == _lib.VBQ_OK             # nothing to do
    assert lib.vbq_swiglu_rows(None, None, 4, 16, 0, None) == _lib.VBQ_ERR_NULL
    assert lib.vbq_swiglu_rows(16, 16, 4, 12, 0, None) == _lib.VBQ_ERR_SHAPE          # n % 8
    assert lib.vbq_swiglu_rows(8, 16, 4, 16, 0, None) == _lib.VBQ_ERR_ALIGN
    assert lib.vbq_moe_sort(None, 10, 8, 2, None, None, None, None) == _lib.VBQ_ERR_NULL
    assert lib.vbq_moe_sort(None, 10, 0, 2, None, None, None, None) == _lib.VBQ_ERR_SHAPE   # E
    assert lib.vbq_moe_sort(None, 10, 5000, 2, None, None, None, None) == _lib.VBQ_ERR_SHAPE
    assert lib.vbq_moe_sort(None, 10, 8, 9, None, None, None, None) == _lib.VBQ_ERR_SHAPE   # topk
    assert b"vbq_moe_sort" in lib.vbq_last_error()


def test_scratch_size_query(lib):
    """Split-K scratch: counters + splits * batch * N partials for the fp32 kernel; none
    when K is tiny, and none for the tensor-core kernels (Q4_K / Q8_0 / Q6_K batch 1..16),
    whose splits add up inside a thread-block cluster."""
    v = C.c_size_t()
    for batch in (1, 2, 3, 4, 5, 8, 16, 32):
        assert lib.vbq_gemv_scratch_bytes(4096, 14336, 14, batch, C.byref(v)) == 0 and v.value == 0
    assert lib.vbq_gemv_scratch_bytes(131072, 1024, 14, 1, C.byref(v)) == 0 and v.value == 0
    # past the Q6_K kernel's K cap the fp32 kernel takes the call, with scratch growing in batch
    assert lib.vbq_gemv_scratch_bytes(131072 + 256, 1024, 14, 1, C.byref(v)) == 0 and v.value > 0
    small = v.value
    assert lib.vbq_gemv_scratch_bytes(131072 + 256, 1024, 14, 16, C.byref(v)) == 0
    assert v.value > small
    for batch in (1, 2, 3, 4, 5, 8, 16):
        assert lib.vbq_gemv_scratch_bytes(4096, 14336, 12, batch, C.byref(v)) == 0 and v.value == 0
    assert lib.vbq_gemv_scratch_bytes(16, 256, 12, 1, C.byref(v)) == 0 and v.value == 0
    assert lib.vbq_gemv_scratch_bytes(4096, 14336, 9, 1, C.byref(v)) == 1
    # past the integer kernels' K cap (exact s32 sums) the fp32 kernel takes the call
    for t in (12, 8):
        assert lib.vbq_gemv_scratch_bytes(3 * 65536, 1024, t, 1, C.byref(v)) == 0 and v.value == 0
        assert lib.vbq_gemv_scratch_bytes(3 * 65536 + 256, 1024, t, 1, C.byref(v)) == 0 and v.value > 0


def test_python_face_rejects_host_tensors():
    import torch
    import vibeblade_b200 as vb
    x = torch.zeros(4096)
    w = torch.zeros(4096 * 144 * 16, dtype=torch.uint8)
    with pytest.raises(RuntimeError, match="CUDA tensors"):
        vb.gemv_dequant(x, w, None, 4096, 4096, "Q4_K")
    with pytest.raises(RuntimeError, match="Unsupported dequant type"):
        vb.gemv_dequant(x, w, None, 4096, 4096, 9)


def test_wait_probe_argument_errors_need_no_gpu(lib):
    from vibeblade_b200 import _lib
    assert lib.vbq_debug_wait_probe(0, 0, None) == _lib.VBQ_ERR_SHAPE
    assert lib.vbq_debug_wait_probe((1 << 31) + 1, 0, None) == _lib.VBQ_ERR_SHAPE
    assert lib.vbq_debug_wait_probe(1000, 2, None) == _lib.VBQ_ERR_SHAPE
    assert b"arrive" in lib.vbq_last_error()


def test_fused_entry_argument_errors_need_no_gpu(lib):
    from vibeblade_b200 import _lib
    assert lib.vbq_gemv_ex(None, None, None, 16, 256, 12, 1, 4, None, None, None, 0, None) == _lib.VBQ_ERR_SHAPE
    assert b"flags" in lib.vbq_last_error()
    assert lib.vbq_gemv_ex(None, None, None, 16, 256, 9, 1, 0, None, None, None, 0, None) == _lib.VBQ_ERR_TYPE
    assert lib.vbq_gemm_ex(None, None, None, 4, 64, 300, 12, 0, None, None, None) == _lib.VBQ_ERR_SHAPE


def test_peer_and_ipc_argument_errors_need_no_gpu(lib):
    """vbq_peer_allreduce and the IPC helpers check their arguments before any CUDA call."""
    from vibeblade_b200 import _lib
    arr = (C.c_void_p * 2)(16, 32)
    assert lib.vbq_peer_allreduce(arr, arr, 0, 0, 1, 8, 64, 0, None) == _lib.VBQ_ERR_SHAPE   # world
    assert lib.vbq_peer_allreduce(arr, arr, 9, 0, 1, 8, 64, 0, None) == _lib.VBQ_ERR_SHAPE
    assert lib.vbq_peer_allreduce(arr, arr, 2, 2, 1, 8, 64, 0, None) == _lib.VBQ_ERR_SHAPE   # rank
    assert lib.vbq_peer_allreduce(arr, arr, 2, 0, 0, 8, 64, 0, None) == _lib.VBQ_ERR_SHAPE   # epoch
    assert lib.vbq_peer_allreduce(arr, arr, 2, 0, 1, -1, 64, 0, None) == _lib.VBQ_ERR_SHAPE  # n
    assert lib.vbq_peer_allreduce(None, arr, 2, 0, 1, 8, 64, 0, None) == _lib.VBQ_ERR_NULL
    bad = (C.c_void_p * 2)(16, 36)  # 36 is not 16-byte aligned
    assert lib.vbq_peer_allreduce(bad, arr, 2, 0, 1, 8, 64, 0, None) == _lib.VBQ_ERR_ALIGN
    assert b"vbq_peer_allreduce" in lib.vbq_last_error()
    assert lib.vbq_ipc_export(None, None, None) == _lib.VBQ_ERR_NULL
    assert lib.vbq_ipc_import(None, 0, None) == _lib.VBQ_ERR_NULL
    assert lib.vbq_ipc_close(None, 0) == _lib.VBQ_ERR_NULL
