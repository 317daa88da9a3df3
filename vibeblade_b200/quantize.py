"""Q4_K / Q6_K / Q8_0 quantizers that write the block layouts the path reads.

The reference ships no GGUF k-quant quantizer (its cpp/src/quantize.cpp and
vibeblade/converter.py write other per-row formats), so these are this library's own:
simple min/max (Q4_K) and abs-max (Q6_K, Q8_0) fits whose output bytes decode with the
reference's dequantizers:

* Q4_K -> ``dequantize_row_q4_K`` (cpp/src/dequant.cpp:258-301), 6-bit scales/mins
  packed the way ``get_scale_min_k4`` unpacks them.
* Q6_K -> ``dequantize_row_q6_K`` (cpp/src/dequant.cpp:359-402): ql nibble i&1 of byte
  i>>1, qh 2-bit field i&3 of byte i>>2, int8 scale per 16 values, fp16 d at byte 208.
* Q8_0 -> the GGUF block: fp16 d then 32 int8 (cpp/src/cuda_kernels.cu:718-735).

Written with torch so the same code runs on host or device tensors.  The arithmetic only
decides which bytes get written; parity between the CUDA path and the reference is
always checked on identical bytes.
"""
from __future__ import annotations

import numpy as np
import torch

from . import formats as F


def _as_tensor(x) -> torch.Tensor:
    if isinstance(x, np.ndarray):
        return torch.from_numpy(np.ascontiguousarray(x, np.float32))
    return x.float().contiguous()


def _f16_bytes(v: torch.Tensor) -> torch.Tensor:
    """fp16 values -> little-endian byte pairs [..., 2] (uint8)."""
    u = v.half().contiguous().view(torch.int16).to(torch.int32) & 0xFFFF
    return torch.stack([u & 0xFF, u >> 8], dim=-1).to(torch.uint8)


def quantize_q8_0(x) -> torch.Tensor:
    x = _as_tensor(x)
    K, N = x.shape
    assert N % 32 == 0, "Q8_0 rows must hold a whole number of 32-value blocks"
    xb = x.reshape(K, N // 32, 32)
    amax = xb.abs().amax(-1)
    d16 = (amax / 127.0).half()
    d = d16.float()
    inv = torch.where(d > 0, 1.0 / d, torch.zeros_like(d))
    q = torch.clamp(torch.round(xb * inv[..., None]), -127, 127).to(torch.int8)
    out = torch.empty(K, N // 32, 34, dtype=torch.uint8, device=x.device)
    out[..., 0:2] = _f16_bytes(d16)
    out[..., 2:34] = q.view(torch.uint8)
    return out.reshape(K, -1)


def _pack_q4k_scales(sc: torch.Tensor, mn: torch.Tensor) -> torch.Tensor:
    """Inverse of get_scale_min_k4 (cpp/src/dequant.cpp:258-266): 8 six-bit scales and 8
    six-bit mins -> 12 bytes."""
    sc = sc.to(torch.int32)
    mn = mn.to(torch.int32)
    out = torch.empty(*sc.shape[:-1], 12, dtype=torch.int32, device=sc.device)
    out[..., 0:4] = (sc[..., 0:4] & 63) | ((sc[..., 4:8] >> 4) << 6)
    out[..., 4:8] = (mn[..., 0:4] & 63) | ((mn[..., 4:8] >> 4) << 6)
    out[..., 8:12] = (sc[..., 4:8] & 0xF) | ((mn[..., 4:8] & 0xF) << 4)
    return out.to(torch.uint8)


def quantize_q4_K(x) -> torch.Tensor:
    x = _as_tensor(x)
    K, N = x.shape
    assert N % 256 == 0, "Q4_K rows must hold a whole number of 256-value blocks"
    nb = N // 256
    xb = x.reshape(K, nb, 8, 32)
    lo = torch.clamp(xb.amin(-1), max=0.0)          # sub-block minimum (<= 0)
    hi = xb.amax(-1)
    step = (hi - lo) / 15.0                          # per sub-block step
    off = -lo                                        # per sub-block offset (>= 0)
    d16 = (step.amax(-1) / 63.0).half()
    dmin16 = (off.amax(-1) / 63.0).half()
    d = d16.float()[..., None]
    dmin = dmin16.float()[..., None]
    sc = torch.where(d > 0, torch.round(step / torch.where(d > 0, d, 1.0)), 0.0).clamp(0, 63)
    mn = torch.where(dmin > 0, torch.round(off / torch.where(dmin > 0, dmin, 1.0)), 0.0).clamp(0, 63)
    eff_step = (d * sc)[..., None]
    eff_off = (dmin * mn)[..., None]
    q = torch.where(eff_step > 0, torch.round((xb + eff_off) / torch.where(eff_step > 0, eff_step, 1.0)),
                    0.0).clamp(0, 15).to(torch.int32)
    # qs byte 32g+l = value 64g+l (low nibble) | value 64g+32+l (high nibble)
    qg = q.reshape(K, nb, 4, 2, 32)
    qs = (qg[..., 0, :] | (qg[..., 1, :] << 4)).reshape(K, nb, 128).to(torch.uint8)
    out = torch.empty(K, nb, 144, dtype=torch.uint8, device=x.device)
    out[..., 0:2] = _f16_bytes(d16)
    out[..., 2:4] = _f16_bytes(dmin16)
    out[..., 4:16] = _pack_q4k_scales(sc, mn)
    out[..., 16:144] = qs
    return out.reshape(K, -1)


def quantize_q6_K(x) -> torch.Tensor:
    x = _as_tensor(x)
    K, N = x.shape
    assert N % 256 == 0, "Q6_K rows must hold a whole number of 256-value blocks"
    nb = N // 256
    xb = x.reshape(K, nb, 16, 16)
    step = xb.abs().amax(-1) / 31.0                  # per 16-value sub-block
    d16 = (step.amax(-1) / 127.0).half()
    d = d16.float()[..., None]
    sc = torch.where(d > 0, torch.round(step / torch.where(d > 0, d, 1.0)), 0.0).clamp(-128, 127)
    eff = (d * sc)[..., None]
    q = torch.where(eff != 0, torch.round(xb / torch.where(eff != 0, eff, 1.0)), 0.0)
    q = (q.clamp(-32, 31) + 32).to(torch.int32).reshape(K, nb, 256)
    lo = q & 0xF
    hi = q >> 4
    ql = (lo[..., 0::2] | (lo[..., 1::2] << 4)).to(torch.uint8)                      # 128 B
    qh = (hi[..., 0::4] | (hi[..., 1::4] << 2) | (hi[..., 2::4] << 4)
          | (hi[..., 3::4] << 6)).to(torch.uint8)                                   # 64 B
    out = torch.empty(K, nb, 210, dtype=torch.uint8, device=x.device)
    out[..., 0:128] = ql
    out[..., 128:192] = qh
    out[..., 192:208] = sc.to(torch.int8).view(torch.uint8)
    out[..., 208:210] = _f16_bytes(d16)
    return out.reshape(K, -1)


_QUANTIZERS = {F.GGML_TYPE_Q8_0: quantize_q8_0, F.GGML_TYPE_Q4_K: quantize_q4_K,
               F.GGML_TYPE_Q6_K: quantize_q6_K}


def quantize(x, qtype) -> torch.Tensor:
    """fp32 [K, N] -> uint8 [K, row_bytes(qtype, N)] in the reference's block layout."""
    return _QUANTIZERS[F.parse_type(qtype)](x)


def synthetic_weights(K: int, N: int, qtype, seed: int = 0, std: float = 0.02,
                      device: str | torch.device = "cpu") -> torch.Tensor:
    """Weights drawn N(0, std) and quantized: the synthetic stand-in for a GGUF tensor.

    On the host the draw uses numpy.random.default_rng(seed); on a device a seeded torch
    generator draws there (faster for the 100 MB-class benchmark matrices)."""
    dev = torch.device(device)
    if dev.type == "cpu":
        w = np.random.default_rng(seed).normal(0.0, std, size=(K, N)).astype(np.float32)
        return quantize(torch.from_numpy(w), qtype)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    w = torch.randn(K, N, generator=g, device=dev, dtype=torch.float32) * std
    return quantize(w, qtype)


# Scale fields of the block types this library reads but does not quantize to: (byte
# offset, fp16 or fp32) per block (cpp/include/ggml_types.h:82-168).
_SCALE_FIELDS = {
    F.GGML_TYPE_Q4_0: [(0, torch.float16)], F.GGML_TYPE_Q4_1: [(0, torch.float16), (2, torch.float16)],
    F.GGML_TYPE_Q5_0: [(0, torch.float16)], F.GGML_TYPE_Q5_1: [(0, torch.float16), (2, torch.float16)],
    F.GGML_TYPE_Q2_K: [(80, torch.float16), (82, torch.float16)], F.GGML_TYPE_Q3_K: [(108, torch.float16)],
    F.GGML_TYPE_Q5_K: [(0, torch.float16), (2, torch.float16)], F.GGML_TYPE_Q8_K: [(0, torch.float32)],
}


def random_block_weights(K: int, N: int, qtype, seed: int = 0, std: float = 1e-3,
                         device: str | torch.device = "cpu") -> torch.Tensor:
    """uint8 [K, row_bytes(qtype, N)] of random code bytes with every scale field drawn
    N(0, std): synthetic weights for the block types without a quantizer here (Q4_0, Q4_1,
    Q5_0, Q5_1, Q2_K, Q3_K, Q5_K, Q8_K).  Their dequantizers are functions of the bytes
    alone, so such weights exercise the same arithmetic and the same bytes per value as a
    file's."""
    t = F.parse_type(qtype)
    if t not in _SCALE_FIELDS:
        raise ValueError(f"random_block_weights: type {t} has a quantizer (use synthetic_weights)")
    bb, bv = F.BLOCK_BYTES[t], F.BLOCK_VALUES[t]
    nb = N // bv
    dev = torch.device(device)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    w = torch.randint(0, 256, (K, nb, bb), generator=g, device=dev, dtype=torch.uint8)
    for off, dt in _SCALE_FIELDS[t]:
        vals = (torch.randn(K, nb, 1, generator=g, device=dev) * std).to(dt)
        w[:, :, off:off + vals.element_size()] = vals.view(torch.uint8)
    return w.reshape(K, nb * bb)
