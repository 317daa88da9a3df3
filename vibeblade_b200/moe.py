"""Mixture-of-experts FFN over quantized expert slabs (device path).

Mirrors the reference's MoE operator (vibeblade/moe.py: ``ExpertRouter.route`` at
:170-206 and ``moe_ffn_silu`` at :407-505; the C++ engine's per-token loop at
cpp/src/fast_model.cpp:534-571, :844-903) with the expert matrices kept as quantized
slabs: the slabs of one projection are packed back to back, slab e at
e * K * row_bytes(type, N) bytes, each a K x N matrix in the reference block layout
(gate / up: K = hidden, N = intermediate; down: K = intermediate, N = hidden).
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from . import formats as F
from .dequant import _require_cuda, _stream_ptr, _weights_u8


def moe_route(logits: torch.Tensor, topk: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Softmax over fp32 logits [T, E] (clipped to +-50), top-k in descending order
    (ties to the lower index), renormalised.  Returns (idx int32 [T, k], weight fp32)."""
    _require_cuda("moe_route", logits)
    if logits.dtype != torch.float32 or logits.dim() != 2:
        raise RuntimeError("moe_route: logits must be fp32 [T, E]")
    T, E = logits.shape
    idx = torch.empty((T, topk), dtype=torch.int32, device=logits.device)
    w = torch.empty((T, topk), dtype=torch.float32, device=logits.device)
    lib = _lib.load()
    _lib.check(lib.vbq_moe_route(logits.data_ptr(), T, E, topk, idx.data_ptr(), w.data_ptr(),
                                 _stream_ptr(logits)), lib)
    return idx, w


def moe_sort(idx: torch.Tensor, E: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Stable counting sort of the (token, slot) entries of idx (int32 [T, topk]) by expert.
    Returns (seg int32 [E + 1], pos int32 [T * topk], tok int32 [T * topk]): expert e owns
    rows seg[e] .. seg[e + 1] - 1, entry j sits at row pos[j] (-1 if its expert is outside
    0..E-1), row r holds token tok[r]; rows of an expert follow entry order."""
    _require_cuda("moe_sort", idx)
    if idx.dtype != torch.int32 or idx.dim() != 2 or not idx.is_contiguous():
        raise RuntimeError("moe_sort: idx must be a contiguous int32 [T, topk] tensor")
    T, k = idx.shape
    seg = torch.empty(E + 1, dtype=torch.int32, device=idx.device)
    pos = torch.empty(T * k, dtype=torch.int32, device=idx.device)
    tok = torch.full((T * k,), -1, dtype=torch.int32, device=idx.device)
    lib = _lib.load()
    _lib.check(lib.vbq_moe_sort(idx.data_ptr(), T, E, k, seg.data_ptr(), pos.data_ptr(),
                                tok.data_ptr(), _stream_ptr(idx)), lib)
    return seg, pos, tok


def gemm_grouped(a: torch.Tensor, slabs: torch.Tensor, seg: torch.Tensor, K: int, N: int, wtype,
                 out: torch.Tensor | None = None, out_dtype=torch.float32,
                 slab_bytes: int | None = None) -> torch.Tensor:
    """Grouped dequant-GEMM: rows seg[s]..seg[s+1] of a (bf16 [rows, K]) times slab s.
    seg is an int32 CUDA tensor of n_seg + 1 offsets."""
    t = F.parse_type(wtype)
    _require_cuda("gemm_grouped", a, slabs, seg)
    if a.dtype != torch.bfloat16 or a.dim() != 2 or a.shape[1] != K:
        raise RuntimeError("gemm_grouped: a must be bf16 [rows, K]")
    if seg.dtype != torch.int32 or seg.dim() != 1 or seg.numel() < 1:
        raise RuntimeError("gemm_grouped: seg must be int32 [n_seg + 1]")
    rows, n_seg = a.shape[0], seg.numel() - 1
    sb = F.matrix_nbytes(t, K, N) if slab_bytes is None else slab_bytes
    w = _weights_u8(slabs)
    if w.numel() < sb * (n_seg - 1) + F.matrix_nbytes(t, K, N):
        raise RuntimeError("gemm_grouped: slabs hold too few bytes for n_seg slabs")
    if out is None:
        out = torch.zeros((rows, N), dtype=out_dtype, device=a.device)
    lib = _lib.load()
    cd = _lib.DTYPE_F32 if out.dtype == torch.float32 else _lib.DTYPE_BF16
    _lib.check(lib.vbq_gemm_grouped(a.data_ptr(), w.data_ptr(), sb, out.data_ptr(), rows, K, N, t,
                                    cd, seg.data_ptr(), n_seg, _stream_ptr(a)), lib)
    return out


_WORKSPACE: dict[tuple[int, int], torch.Tensor] = {}


def moe_workspace_bytes(T: int, H: int, I: int, E: int, topk: int) -> int:
    lib = _lib.load()
    v = C.c_size_t()
    _lib.check(lib.vbq_moe_workspace_bytes(T, H, I, E, topk, C.byref(v)), lib)
    return int(v.value)


def moe_ffn(x: torch.Tensor, logits: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor,
            w_down: torch.Tensor, I: int, wtype, topk: int = 2, out: torch.Tensor | None = None,
            type_up=None, type_down=None, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """out[t] = sum over the top-k experts e of w[t,e] * down_e(silu(gate_e x[t]) * up_e x[t]).

    x fp32 [T, H], logits fp32 [T, E]; w_gate / w_up / w_down the packed expert slabs.
    A workspace is cached per (device, stream) when none is given."""
    tg = F.parse_type(wtype)
    tu = tg if type_up is None else F.parse_type(type_up)
    td = tg if type_down is None else F.parse_type(type_down)
    _require_cuda("moe_ffn", x, logits, w_gate, w_up, w_down)
    if x.dtype != torch.float32 or x.dim() != 2 or logits.dtype != torch.float32 or logits.dim() != 2:
        raise RuntimeError("moe_ffn: x must be fp32 [T, H] and logits fp32 [T, E]")
    T, H = x.shape
    E = logits.shape[1]
    if logits.shape[0] != T:
        raise RuntimeError("moe_ffn: x and logits disagree on T")
    for name, w, t, k, n in (("gate", w_gate, tg, H, I), ("up", w_up, tu, H, I),
                             ("down", w_down, td, I, H)):
        if _weights_u8(w).numel() < E * F.matrix_nbytes(t, k, n):
            raise RuntimeError(f"moe_ffn: {name} slabs hold too few bytes for {E} experts")
    if out is None:
        out = torch.empty((T, H), dtype=torch.float32, device=x.device)
    need = moe_workspace_bytes(T, H, I, E, topk)
    if workspace is None:
        key = (x.device.index or 0, _stream_ptr(x))
        workspace = _WORKSPACE.get(key)
        if workspace is None or workspace.numel() < need:
            workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
            _WORKSPACE[key] = workspace
    lib = _lib.load()
    _lib.check(lib.vbq_moe_ffn(x.data_ptr(), logits.data_ptr(), _weights_u8(w_gate).data_ptr(),
                               _weights_u8(w_up).data_ptr(), _weights_u8(w_down).data_ptr(),
                               out.data_ptr(), T, H, I, E, topk, tg, tu, td, workspace.data_ptr(),
                               workspace.numel(), _stream_ptr(x)), lib)
    return out
