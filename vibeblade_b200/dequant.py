"""Python face of the device k-quant path, mirroring the reference's operator API.

Names, argument order and error text follow ``cpp/include/dequant.h:11-48``
(``dequantize_row``, ``gemv_dequant``, ``gemv_dequant_mt``) with torch CUDA tensors in
place of raw pointers, so call sites such as ``forward_layer``'s
``gemv_dequant(x, W, out, K, N, type, scratch)`` (cpp/src/fast_model.cpp:655-657) swap over
unchanged.  All work runs in libvbq.so (sm_100a) on the current torch stream; there is no
CPU fallback.
"""
from __future__ import annotations

import torch

from . import _lib
from . import formats as F


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream_ptr(t: torch.Tensor) -> int:
    """The current CUDA stream of t's device as a raw handle (no Stream object per call:
    this runs once per operator call on the decode path)."""
    if _raw_stream is not None:
        return _raw_stream(t.device.index if t.device.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(t.device).cuda_stream


def _require_cuda(name: str, *ts: torch.Tensor) -> None:
    for t in ts:
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise RuntimeError(f"{name}: tensors must be CUDA tensors (the k-quant path runs on "
                               "the GPU only)")
        if not t.is_contiguous():
            raise RuntimeError(f"{name}: tensors must be contiguous")


def _weights_u8(w: torch.Tensor) -> torch.Tensor:
    return w if w.dtype == torch.uint8 else w.view(torch.uint8)


# Zero-filled split-K scratch per (device, stream).  Calls on one stream run in order,
# and every call leaves the buffer zero-filled again, so one buffer per stream is safe.
_SCRATCH: dict[tuple[int, int], torch.Tensor] = {}


_CUDA_AVAILABLE: list[bool] = []


def _cuda_available() -> bool:
    if not _CUDA_AVAILABLE:
        _CUDA_AVAILABLE.append(torch.cuda.is_available())
    return _CUDA_AVAILABLE[0]


# scratch sizes per (device, K, N, type, batch): the plan depends on the device's SM count
_SCRATCH_BYTES: dict[tuple[int, int, int, int, int], int] = {}
# validated gemv_dequant calls: (type as given, K, N, x values, device index) -> (type id,
# batch, weight bytes needed, scratch bytes)
_GEMV_PLANS: dict[tuple, tuple[int, int, int, int]] = {}


def gemv_scratch_bytes(K: int, N: int, wtype, batch: int = 1) -> int:
    """Bytes of scratch ``gemv_dequant`` needs for this shape on the current device."""
    t = F.parse_type(wtype)
    dev = torch.cuda.current_device() if _cuda_available() else -1
    key = (dev, K, N, t, batch)
    hit = _SCRATCH_BYTES.get(key)
    if hit is not None:
        return hit
    import ctypes as C
    lib = _lib.load()
    v = C.c_size_t()
    _lib.check(lib.vbq_gemv_scratch_bytes(K, N, t, batch, C.byref(v)), lib)
    _SCRATCH_BYTES[key] = int(v.value)
    return int(v.value)


def _stream_scratch(device: torch.device, stream: int, nbytes: int) -> torch.Tensor:
    key = (device.index if device.index is not None else torch.cuda.current_device(), stream)
    buf = _SCRATCH.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _SCRATCH[key] = buf
    return buf


def row_bytes(qtype, n: int) -> int:
    """Bytes per row of a K x N matrix (cpp/src/dequant.cpp:749-763)."""
    return F.row_bytes(qtype, n)


def dequantize(weights: torch.Tensor, K: int, N: int, wtype, dtype=torch.float32,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """Dequantize a K x N quantized matrix to fp32 (bit-exact with the reference's
    dequantize_row, row by row) or bf16 (that value rounded to nearest-even)."""
    t = F.parse_type(wtype)
    _require_cuda("dequantize", weights)
    if dtype not in (torch.float32, torch.bfloat16):
        raise RuntimeError("dequantize: dtype must be torch.float32 or torch.bfloat16")
    w = _weights_u8(weights)
    need = F.row_bytes(t, N) * K if K > 1 else F.tensor_nbytes(t, N)
    if w.numel() < need:
        raise RuntimeError(f"dequantize: weights hold {w.numel()} bytes, need {need}")
    if out is None:
        out = torch.empty((K, N), dtype=dtype, device=w.device)
    else:
        _require_cuda("dequantize", out)
        if out.dtype != dtype or out.numel() < K * N:
            raise RuntimeError("dequantize: out has the wrong dtype or size")
    lib = _lib.load()
    od = _lib.DTYPE_F32 if dtype == torch.float32 else _lib.DTYPE_BF16
    _lib.check(lib.vbq_dequantize(w.data_ptr(), out.data_ptr(), K, N, t, od, _stream_ptr(w)), lib)
    return out


def dequantize_row(row: torch.Tensor, out: torch.Tensor | None, n_values: int, type) -> torch.Tensor:
    """``void dequantize_row(const void* row, float* out, int64_t n, ggml_type)``
    (cpp/include/dequant.h:11): n_values may be ragged; returns ``out`` (allocated when
    None) holding n_values fp32 values."""
    res = dequantize(row, 1, n_values, type, torch.float32,
                     None if out is None else out.view(1, -1))
    return res.view(-1)[:n_values]


def gemv_dequant(x: torch.Tensor, weights: torch.Tensor, out: torch.Tensor | None, K: int,
                 N: int, wtype, scratch: torch.Tensor | None = None) -> torch.Tensor:
    """``gemv_dequant(x, W, out, K, N, wtype, scratch)`` (cpp/include/dequant.h:27-35):
    out[n] = sum_k x[k] * deq(W)[k, n].

    ``x`` may also be a batch [B, K] with B <= 32 (the reference engine makes B calls,
    cpp/src/fast_model.cpp:645-660); ``out`` is then [B, N].  ``scratch`` is the
    caller-owned split-K buffer, as in the reference: a CUDA tensor of at least
    ``gemv_scratch_bytes(K, N, wtype, B)`` bytes, zero-filled before its first use (each
    call leaves it zero-filled).  When None, a per-stream buffer owned by this module is
    used."""
    # Decode fast path: a call shaped like an earlier validated one (same type, K, N, x size
    # and device) needs only the per-tensor checks; anything unusual takes the full path
    # below, which raises the reference's errors.
    plan = _GEMV_PLANS.get((wtype, K, N, x.numel(), x.device.index)) if isinstance(x, torch.Tensor) else None
    if (plan is not None and x.is_cuda and x.dtype == torch.float32 and x.is_contiguous()
            and isinstance(weights, torch.Tensor) and weights.is_cuda and weights.is_contiguous()
            and isinstance(out, torch.Tensor) and out.is_cuda and out.dtype == torch.float32
            and out.is_contiguous() and scratch is None):
        t, batch, need_w, need_s = plan
        w = weights if weights.dtype == torch.uint8 else weights.view(torch.uint8)
        if w.numel() >= need_w and out.numel() == batch * N:
            sp = _stream_ptr(x)
            scr = _stream_scratch(x.device, sp, need_s) if need_s else None
            lib = _lib.load()
            _lib.check(lib.vbq_gemv(x.data_ptr(), w.data_ptr(), out.data_ptr(), K, N, t, batch,
                                    scr.data_ptr() if scr is not None else None,
                                    scr.numel() if scr is not None else 0, sp), lib)
            return out
    t = F.parse_type(wtype)
    _require_cuda("gemv_dequant", x, weights)
    if x.dtype != torch.float32:
        raise RuntimeError("gemv_dequant: x must be float32")
    if K > 0:
        if x.numel() % K != 0:
            raise RuntimeError(f"gemv_dequant: x has {x.numel()} values, not a multiple of K={K}")
        batch = x.numel() // K
    else:
        batch = x.shape[0] if x.dim() > 1 else 1
    generic = t not in F.QUANTIZED or N % 256 != 0  # the generic kernel: any batch
    limit = 4 * 65535 if generic else 32
    if not 1 <= batch <= limit:
        raise RuntimeError(f"gemv_dequant: batch must be in 1..{limit}, got {batch}")
    w = _weights_u8(weights)
    need = F.row_bytes(t, N) * K
    if w.numel() < need:
        raise RuntimeError(f"gemv_dequant: weights hold {w.numel()} bytes, need {need}")
    if out is None:
        out = torch.empty((batch, N) if x.dim() > 1 else (N,), dtype=torch.float32, device=x.device)
    else:
        _require_cuda("gemv_dequant", out)
        if out.dtype != torch.float32 or out.numel() != batch * N:
            raise RuntimeError("gemv_dequant: out must be float32 with batch*N values")
    lib = _lib.load()
    sp = _stream_ptr(x)
    need = gemv_scratch_bytes(K, N, t, batch) if K > 0 else 0
    if scratch is None:
        scr = _stream_scratch(x.device, sp, need) if need else None
    else:
        _require_cuda("gemv_dequant", scratch)
        scr = scratch
    scr_ptr = scr.data_ptr() if scr is not None else None
    scr_bytes = scr.numel() * scr.element_size() if scr is not None else 0
    _lib.check(lib.vbq_gemv(x.data_ptr(), w.data_ptr(), out.data_ptr(), K, N, t, batch,
                            scr_ptr, scr_bytes, sp), lib)
    if K > 0 and len(_GEMV_PLANS) < 4096:
        _GEMV_PLANS[(wtype, K, N, x.numel(), x.device.index)] = (t, batch, F.row_bytes(t, N) * K, need)
    return out


def gemv_dequant_mt(x: torch.Tensor, weights: torch.Tensor, out: torch.Tensor | None, K: int,
                    N: int, wtype, n_threads: int = 0,
                    scratch: torch.Tensor | None = None) -> torch.Tensor:
    """``gemv_dequant_mt`` (cpp/include/dequant.h:39-48).  The reference ignores
    n_threads; here the whole GPU runs the call, so it is ignored as well."""
    return gemv_dequant(x, weights, out, K, N, wtype, scratch)


def gemv_fused(x: torch.Tensor, weights: torch.Tensor, out: torch.Tensor | None, K: int, N: int,
               wtype, bias: torch.Tensor | None = None, residual: torch.Tensor | None = None,
               swiglu_input: bool = False, scratch: torch.Tensor | None = None) -> torch.Tensor:
    """``gemv_dequant`` with the element-wise steps around it fused in (vbq_gemv_ex):

    * ``swiglu_input``: ``x`` is [B, 2K], the output of a gate | up matmul, and the GEMV's
      input is silu(gate) * up (cpp/src/fast_model.cpp:946-953) -- the down projection
      without a SwiGLU pass;
    * ``bias`` fp32 [N] is added to every row (Q/K/V biases, :659-668);
    * ``residual`` fp32 [B, N] is added as well (the residual adds after o and down); it may
      be ``out`` itself for an in-place update.
    """
    t = F.parse_type(wtype)
    _require_cuda("gemv_fused", x, weights)
    if x.dtype != torch.float32:
        raise RuntimeError("gemv_fused: x must be float32")
    kx = 2 * K if swiglu_input else K
    if K <= 0 or x.numel() % kx != 0:
        raise RuntimeError(f"gemv_fused: x has {x.numel()} values, not a multiple of {kx}")
    batch = x.numel() // kx
    w = _weights_u8(weights)
    if w.numel() < F.row_bytes(t, N) * K:
        raise RuntimeError(f"gemv_fused: weights hold {w.numel()} bytes, need {F.row_bytes(t, N) * K}")
    for name, v, n in (("bias", bias, N), ("residual", residual, batch * N)):
        if v is not None:
            _require_cuda("gemv_fused", v)
            if v.dtype != torch.float32 or v.numel() != n:
                raise RuntimeError(f"gemv_fused: {name} must be float32 with {n} values")
    if out is None:
        out = torch.empty((batch, N), dtype=torch.float32, device=x.device)
    else:
        _require_cuda("gemv_fused", out)
        if out.dtype != torch.float32 or out.numel() != batch * N:
            raise RuntimeError("gemv_fused: out must be float32 with batch*N values")
    lib = _lib.load()
    sp = _stream_ptr(x)
    need = gemv_scratch_bytes(K, N, t, batch)
    scr = (_stream_scratch(x.device, sp, need) if need else None) if scratch is None else scratch
    _lib.check(lib.vbq_gemv_ex(x.data_ptr(), w.data_ptr(), out.data_ptr(), K, N, t, batch,
                               1 if swiglu_input else 0,
                               bias.data_ptr() if bias is not None else None,
                               residual.data_ptr() if residual is not None else None,
                               scr.data_ptr() if scr is not None else None,
                               scr.numel() * scr.element_size() if scr is not None else 0, sp), lib)
    return out
