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


def gemm_swiglu(a: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor, out: torch.Tensor | None,
                M: int, K: int, I: int, wtype, row_bytes: int = 0) -> torch.Tensor:
    """The gate | up GEMM fused with SwiGLU (vbq_gemm_swiglu): bf16 [M, I] =
    silu(a W_gate) * (a W_up) (cpp/src/fast_model.cpp:906-953), the same bits as two
    ``gemm_dequant`` calls with bf16 output and ``swiglu`` without the [M, 2I] round trip.

    ``a``: bf16 [M, K]; ``w_gate`` / ``w_up``: the block bytes of two K x I matrices of one
    type, each starting at its tensor's data pointer with rows ``row_bytes`` apart (0: the
    packed row of I columns).  For a gate | up matrix packed side by side, pass it as
    ``w_gate``, ``w_up`` = a view starting at the up part, and the packed row stride."""
    t = F.parse_type(wtype)
    _require_cuda("gemm_swiglu", a)
    for w in (w_gate, w_up):
        if not isinstance(w, torch.Tensor) or not w.is_cuda:
            raise RuntimeError("gemm_swiglu: tensors must be CUDA tensors (the k-quant path runs on the GPU only)")
    if a.dtype != torch.bfloat16 or a.numel() != M * K:
        raise RuntimeError(f"gemm_swiglu: a must be bfloat16 with M*K = {M * K} values")
    stride = row_bytes or F.row_bytes(t, I)
    for name, w in (("w_gate", w_gate), ("w_up", w_up)):
        span = w.numel() * w.element_size() if w.is_contiguous() else None
        if span is not None and K > 0 and span < stride * (K - 1) + F.row_bytes(t, I):
            raise RuntimeError(f"gemm_swiglu: {name} holds {span} bytes, too few for {K} rows")
    if out is None:
        out = torch.empty((M, I), dtype=torch.bfloat16, device=a.device)
    else:
        _require_cuda("gemm_swiglu", out)
        if out.dtype != torch.bfloat16 or out.numel() != M * I:
            raise RuntimeError("gemm_swiglu: out must be bfloat16 with M*I values")
    lib = _lib.load()
    _lib.check(lib.vbq_gemm_swiglu(a.data_ptr(), w_gate.data_ptr(), w_up.data_ptr(), out.data_ptr(), M, K, I,
                                   t, row_bytes, _stream_ptr(a)), lib)
    return out
