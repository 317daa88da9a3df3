"""Device-side failure detection without a GPU fault.

Every wait inside the library's kernels is bounded; when one runs out the kernel records
a status bit, finishes normally, and vbq_device_status reports VBQ_ERR_TIMEOUT (the
reference's CUDA path throws on the host instead, cpp/src/cuda_kernels.cu:24-40).  The
diagnostic entry vbq_debug_wait_probe runs that same wait on a barrier nothing arrives
on, with a budget of a few milliseconds, so the report path is exercised without a hang:
the status is raised, read, cleared, and the context keeps working afterwards.
"""
from __future__ import annotations

import ctypes as C

import pytest
import torch

import vibeblade_b200 as vb
from vibeblade_b200 import _lib
from vibeblade_b200.quantize import synthetic_weights

pytestmark = pytest.mark.gpu

BUDGET = 4_000_000  # SM cycles, about 2 ms at 1.965 GHz


def _status(lib, clear):
    v = C.c_int32(-1)
    rc = lib.vbq_device_status(C.byref(v), 1 if clear else 0)
    return rc, int(v.value)


def test_wait_probe_reports_timeout_then_clears(cuda):
    lib = _lib.load()
    stream = torch.cuda.current_stream(cuda).cuda_stream
    torch.cuda.synchronize()
    assert _status(lib, True)[0] in (_lib.VBQ_OK, _lib.VBQ_ERR_TIMEOUT)  # start clean
    # the wait succeeds when the phase completes: no status
    _lib.check(lib.vbq_debug_wait_probe(BUDGET, 1, stream), lib)
    torch.cuda.synchronize()
    assert _status(lib, False) == (_lib.VBQ_OK, 0)
    # nothing arrives: the wait gives up, the kernel returns, the status says timeout
    _lib.check(lib.vbq_debug_wait_probe(BUDGET, 0, stream), lib)
    torch.cuda.synchronize()
    rc, st = _status(lib, False)
    assert rc == _lib.VBQ_ERR_TIMEOUT and st & 1
    assert b"bounded device-side wait" in lib.vbq_last_error()
    # the bit is sticky until cleared, then reads clean
    rc, st = _status(lib, True)
    assert rc == _lib.VBQ_ERR_TIMEOUT and st & 1
    assert _status(lib, False) == (_lib.VBQ_OK, 0)


def test_context_usable_after_a_timeout(cuda):
    """After a wait ran out, the same process keeps computing correct results."""
    lib = _lib.load()
    stream = torch.cuda.current_stream(cuda).cuda_stream
    _lib.check(lib.vbq_debug_wait_probe(BUDGET, 0, stream), lib)
    torch.cuda.synchronize()
    assert vb.device_status(clear=True) & 1
    K, N, t = 4096, 4096, 12
    w = synthetic_weights(K, N, t, seed=5, device=cuda)
    x = torch.randn(2, K, device=cuda)
    y = vb.gemv_dequant(x, w, None, K, N, t)
    ref = x.double() @ vb.dequantize(w, K, N, t).double()
    assert ((y.double() - ref).abs().max() / ref.abs().max()).item() <= 1e-3
    assert vb.device_status() == 0
