"""Quantized-weight GEMM (prefill) on the tcgen05 tensor cores.

The reference runs prefill as one ``gemv_dequant`` per token
(cpp/src/fast_model.cpp:645-660); ``gemm_dequant`` computes all tokens at once:
out[m, n] = sum_k a[m, k] * deq(W)[k, n], with a in bf16 and fp32 accumulation.
"""
from __future__ import annotations

import torch

from . import _lib
from . import formats as F
from .dequant import _require_cuda, _stream_ptr, _weights_u8


def gemm_dequant(a: torch.Tensor, weights: torch.Tensor, out: torch.Tensor | None, M: int,
                 K: int, N: int, wtype, out_dtype=torch.float32, bias: torch.Tensor | None = None,
                 residual: torch.Tensor | None = None) -> torch.Tensor:
    """a: bf16 [M, K] CUDA tensor; weights: the K x N block bytes; returns [M, N] in
    out_dtype (torch.float32 or torch.bfloat16).  Optional epilogue (vbq_gemm_ex): ``bias``
    fp32 [N] and ``residual`` [M, N] of out_dtype (may be ``out`` itself) are added to the
    fp32 accumulator before the one rounding to out_dtype."""
    t = F.parse_type(wtype)
    _require_cuda("gemm_dequant", a, weights)
    if a.dtype != torch.bfloat16:
        raise RuntimeError("gemm_dequant: a must be bfloat16")
    if a.numel() != M * K:
        raise RuntimeError(f"gemm_dequant: a has {a.numel()} values, expected M*K = {M * K}")
    if out_dtype not in (torch.float32, torch.bfloat16):
        raise RuntimeError("gemm_dequant: out_dtype must be torch.float32 or torch.bfloat16")
    w = _weights_u8(weights)
    need = F.row_bytes(t, N) * K
    if w.numel() < need:
        raise RuntimeError(f"gemm_dequant: weights hold {w.numel()} bytes, need {need}")
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=a.device)
    else:
        _require_cuda("gemm_dequant", out)
        if out.dtype != out_dtype or out.numel() != M * N:
            raise RuntimeError("gemm_dequant: out has the wrong dtype or size")
    lib = _lib.load()
    cd = _lib.DTYPE_F32 if out_dtype == torch.float32 else _lib.DTYPE_BF16
    if bias is None and residual is None:
        _lib.check(lib.vbq_gemm(a.data_ptr(), w.data_ptr(), out.data_ptr(), M, K, N, t, cd,
                                _stream_ptr(a)), lib)
        return out
    if bias is not None:
        _require_cuda("gemm_dequant", bias)
        if bias.dtype != torch.float32 or bias.numel() != N:
            raise RuntimeError("gemm_dequant: bias must be float32 [N]")
    if residual is not None:
        _require_cuda("gemm_dequant", residual)
        if residual.dtype != out_dtype or residual.numel() != M * N:
            raise RuntimeError("gemm_dequant: residual must be [M, N] of out_dtype")
    _lib.check(lib.vbq_gemm_ex(a.data_ptr(), w.data_ptr(), out.data_ptr(), M, K, N, t, cd,
                               bias.data_ptr() if bias is not None else None,
                               residual.data_ptr() if residual is not None else None,
                               _stream_ptr(a)), lib)
    return out


def device_status(clear: bool = True) -> int:
    """Device-side status bits (1 = a bounded wait inside a kernel gave up)."""
    import ctypes as C
    lib = _lib.load()
    v = C.c_int32()
    rc = lib.vbq_device_status(C.byref(v), 1 if clear else 0)
    if rc not in (_lib.VBQ_OK, _lib.VBQ_ERR_TIMEOUT):
        _lib.check(rc, lib)
    return int(v.value)
