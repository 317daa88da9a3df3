"""The allocation-free GEMV entry point, vbq_gemv_static_scratch.

It serves callers that cannot allocate device memory (an engine that reserved all of
HBM for its own pools, a plugin that only receives the host's buffers) by keeping the
split-K scratch in a fixed array inside the library.  Checked through the C ABI against
vbq_gemv with caller-owned scratch, twice in a row on each shape, because the array is
shared by every call and keeps the previous call's contents.

This file sorts last so that a run stopping at the first failure has run everything else.
"""
from __future__ import annotations

import ctypes as C

import pytest
import torch

from vibeblade_b200 import _lib
from vibeblade_b200.quantize import synthetic_weights

pytestmark = pytest.mark.gpu

TOL = 1e-3  # max-norm relative error, as in the other GEMV tests

SHAPES = [
    (12, 4096, 14336, 1),    # Q4_K gate/up of the decode layer (cluster split-K, no scratch)
    (12, 14336, 4096, 4),    # Q4_K down, batch 4
    (8, 8192, 10240, 16),    # Q8_0 70B-shape QKV, batch 16
    (12, 300, 1024, 3),      # ragged K: a single split, no scratch at all
    (14, 4096, 4096, 24),    # Q6_K batch 24: groups of 4 rows on the tensor-core kernel
    # K past the tensor-core kernels' caps: the fp32 kernel, its split-K scratch in the array
    (14, 131328, 1024, 2),   # Q6_K (cap 2^17)
    (12, 196864, 512, 3),    # Q4_K (cap 3 x 2^16)
]


def _scratch_bytes(lib, K, N, t, B) -> int:
    v = C.c_size_t()
    _lib.check(lib.vbq_gemv_scratch_bytes(K, N, t, B, C.byref(v)), lib)
    return int(v.value)


@pytest.mark.parametrize("t,K,N,B", SHAPES)
def test_static_scratch_matches_vbq_gemv_twice(cuda, t, K, N, B):
    lib = _lib.load()
    stream = torch.cuda.current_stream(cuda).cuda_stream
    w = synthetic_weights(K, N, t, seed=7, device=cuda)
    g = torch.Generator(device=cuda).manual_seed(11)
    need = _scratch_bytes(lib, K, N, t, B)
    scratch = torch.zeros(max(need, 16), dtype=torch.uint8, device=cuda)
    for call in range(2):
        x = torch.randn(B, K, generator=g, device=cuda)
        y_ref = torch.empty(B, N, device=cuda)
        _lib.check(lib.vbq_gemv(x.data_ptr(), w.data_ptr(), y_ref.data_ptr(), K, N, t, B,
                                scratch.data_ptr(), scratch.numel(), stream), lib)
        y = torch.full((B, N), float("nan"), device=cuda)
        _lib.check(lib.vbq_gemv_static_scratch(x.data_ptr(), w.data_ptr(), y.data_ptr(), K, N,
                                               t, B, stream), lib)
        torch.cuda.synchronize()
        assert torch.isfinite(y).all(), f"call {call}: output not fully written"
        err = ((y.double() - y_ref.double()).abs().max() / y_ref.double().abs().max()).item()
        assert err <= TOL, f"call {call}: max-norm relative error {err}"


_REJECT_SCRIPT = r"""
import ctypes as C, sys, torch
sys.path.insert(0, sys.argv[1])
from vibeblade_b200 import _lib
lib = _lib.load()
K, N, t, B = 4096, 14336, 14, 16  # Q6_K on the fp32 split-K kernel (VBQ_GEMV_SCALAR=1)
v = C.c_size_t()
assert lib.vbq_gemv_scratch_bytes(K, N, t, B, C.byref(v)) == 0
assert v.value > (8 << 20), v.value
x = torch.zeros(B, K, device="cuda")
w = torch.zeros(K * (N // 256) * 210, dtype=torch.uint8, device="cuda")
y = torch.zeros(B, N, device="cuda")
rc = lib.vbq_gemv_static_scratch(x.data_ptr(), w.data_ptr(), y.data_ptr(), K, N, t, B,
                                 torch.cuda.current_stream().cuda_stream)
assert rc == _lib.VBQ_ERR_WORKSPACE, rc
assert b"fixed" in lib.vbq_last_error()
print("rejected")
"""


def test_static_scratch_rejects_shapes_beyond_its_size(cuda):
    """The split planner keeps scratch to a few MB, inside the fixed array; a tuning
    override of the split factor (VBQ_GEMV_SPLIT, read once per process, hence the child
    process; VBQ_GEMV_SCALAR=1 keeps the shape on the fp32 kernel, the one that uses
    scratch) makes a shape need more, and the call must refuse it without launching."""
    import os
    import subprocess
    import sys
    from pathlib import Path
    root = str(Path(__file__).resolve().parents[1])
    env = dict(os.environ, VBQ_GEMV_SPLIT="64", VBQ_GEMV_SCALAR="1")
    r = subprocess.run([sys.executable, "-c", _REJECT_SCRIPT, root], env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "rejected" in r.stdout, r.stdout + r.stderr


_SCALAR_SCRIPT = r"""
import ctypes as C, sys, torch
sys.path.insert(0, sys.argv[1])
from vibeblade_b200 import _lib
from vibeblade_b200.quantize import synthetic_weights
lib = _lib.load()
dev = torch.device("cuda", 0)
stream = torch.cuda.current_stream(dev).cuda_stream
g = torch.Generator(device=dev).manual_seed(13)
for t, K, N, B in [(12, 4096, 14336, 1), (12, 14336, 4096, 20), (8, 8192, 10240, 4)]:
    v = C.c_size_t()
    assert lib.vbq_gemv_scratch_bytes(K, N, t, B, C.byref(v)) == 0
    assert v.value > 0, (t, K, N, B)  # the scratch-using kernel is the one under test
    w = synthetic_weights(K, N, t, seed=17, device=dev)
    scratch = torch.zeros(v.value, dtype=torch.uint8, device=dev)
    for call in range(2):
        x = torch.randn(B, K, generator=g, device=dev)
        y_ref = torch.empty(B, N, device=dev)
        assert lib.vbq_gemv(x.data_ptr(), w.data_ptr(), y_ref.data_ptr(), K, N, t, B,
                            scratch.data_ptr(), scratch.numel(), stream) == 0
        y = torch.full((B, N), float("nan"), device=dev)
        rc = lib.vbq_gemv_static_scratch(x.data_ptr(), w.data_ptr(), y.data_ptr(), K, N, t, B, stream)
        assert rc == 0, lib.vbq_last_error()
        torch.cuda.synchronize()
        assert torch.isfinite(y).all(), (t, call)
        err = ((y.double() - y_ref.double()).abs().max() / y_ref.double().abs().max()).item()
        assert err <= 1e-3, (t, call, err)
print("scalar ok")
"""


def test_static_scratch_on_the_split_k_kernel_for_all_types(cuda):
    """Q4_K and Q8_0 normally run on tensor-core kernels that need no scratch; the
    comparison switch VBQ_GEMV_SCALAR=1 (read once per process, hence the child process)
    sends them to the split-K kernel, so the array is used for every type, twice per shape
    (batch 20 also as two launches)."""
    import os
    import subprocess
    import sys
    from pathlib import Path
    root = str(Path(__file__).resolve().parents[1])
    env = dict(os.environ, VBQ_GEMV_SCALAR="1")
    r = subprocess.run([sys.executable, "-c", _SCALAR_SCRIPT, root], env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "scalar ok" in r.stdout, r.stdout + r.stderr
