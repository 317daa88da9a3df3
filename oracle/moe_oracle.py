"""CPU restatement of the reference's MoE FFN (TEST INFRASTRUCTURE ONLY).

Only tests/ and the bench's CPU-baseline leg use this module, as the checker; the product
path (vibeblade_b200.moe) never calls it.

Follows vibeblade/moe.py:
* ``route``: ExpertRouter.route after its matmul (:183-206): logits clipped to +-50,
  softmax (:84-88), top-k, weights renormalised (sum < 1e-12 -> 1).  The reference picks
  the top k with argpartition, which leaves the order of the k winners (and ties)
  unspecified; this restatement orders them by descending probability, ties to the lower
  expert index, the order the device kernel uses.
* ``moe_ffn``: moe_ffn_silu (:407-505) without a shared expert: per slot k,
  gate = x Wg_e, up = x Wu_e, both sanitised (nan -> 0, clip +-65504), hidden =
  silu(gate) * up (silu as :36-50), out_k = hidden Wd_e; moe_out += w_k * out_k in slot
  order; output sanitised.
``mode="fp32"`` evaluates it in float32 like the reference; ``mode="device"`` evaluates in
float64 but rounds x, the projections and the SwiGLU product to bf16 where the device path
does, which isolates accumulation-order error when comparing against the GPU.
"""
from __future__ import annotations

import numpy as np


def _bf16(a: np.ndarray) -> np.ndarray:
    """Round float32 values to bfloat16 (nearest-even), returned as float32."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    nan = np.isnan(a)
    out = r.view(np.float32).copy()
    out[nan] = np.nan
    return out


def softmax32(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    m = np.max(x, axis=-1, keepdims=True)
    e = np.exp(x - m)
    return e / np.sum(e, axis=-1, keepdims=True)


def route(logits: np.ndarray, topk: int) -> tuple[np.ndarray, np.ndarray]:
    lg = np.clip(np.asarray(logits, dtype=np.float32), -50.0, 50.0)
    probs = softmax32(lg)
    T, E = probs.shape
    # stable sort of -p: descending probability, ties in index order
    order = np.argsort(-probs, axis=-1, kind="stable")[:, :topk]
    w = np.take_along_axis(probs, order, axis=-1)
    s = w.sum(axis=-1, keepdims=True)
    s = np.where(s < 1e-12, 1.0, s)
    return order.astype(np.int32), (w / s).astype(np.float32)


def _sanitize(a: np.ndarray) -> np.ndarray:
    return np.clip(np.nan_to_num(a, nan=0.0, posinf=65504.0, neginf=-65504.0), -65504.0, 65504.0)


def silu(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x)
    with np.errstate(over="ignore", invalid="ignore"):
        pos = x >= 0
        s = np.empty_like(x)
        s[pos] = 1.0 / (1.0 + np.exp(-x[pos]))
        ep = np.exp(x[~pos])
        s[~pos] = ep / (1.0 + ep)
    s = np.nan_to_num(s, nan=0.0, posinf=1.0, neginf=0.0)
    return x * s


def moe_ffn(x: np.ndarray, logits: np.ndarray, wg: np.ndarray, wu: np.ndarray, wd: np.ndarray,
            topk: int, mode: str = "fp32") -> np.ndarray:
    """x [T, H]; wg, wu [E, H, I]; wd [E, I, H] (dense, already dequantized)."""
    idx, w = route(logits, topk)
    if mode == "fp32":
        dt = np.float32
        xx = np.asarray(x, dtype=np.float32)
        rnd = lambda a: a  # noqa: E731
    elif mode == "device":
        dt = np.float64
        xx = _bf16(np.asarray(x, dtype=np.float32)).astype(np.float64)
        rnd = lambda a: _bf16(a.astype(np.float32)).astype(np.float64)  # noqa: E731
    else:
        raise ValueError(mode)
    T, H = xx.shape
    out = np.zeros((T, H), dtype=dt)
    for k in range(topk):
        for e in np.unique(idx[:, k]):
            rows = np.nonzero(idx[:, k] == e)[0]
            xe = xx[rows]
            g = rnd(_sanitize(xe @ wg[e].astype(dt)))
            u = rnd(_sanitize(xe @ wu[e].astype(dt)))
            h = rnd(silu(g) * u) if mode == "device" else silu(g) * u
            y = h @ wd[e].astype(dt)
            if mode == "device":
                y = y.astype(np.float32).astype(np.float64)
            out[rows] = out[rows] + w[rows, k:k + 1].astype(dt) * y
    return _sanitize(out).astype(np.float32)
