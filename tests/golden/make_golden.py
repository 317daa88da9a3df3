"""Generate the golden vectors in tests/golden/*.npz from the reference itself.

Run where the reference checkout is mounted (``$VB_REF`` names it; build.py holds the default):

    python tests/golden/make_golden.py

Sources of truth:
* Q4_K and Q6_K dequant + gemv: the reference's own ``vibeblade::dequantize_row`` and
  ``vibeblade::gemv_dequant`` (cpp/src/dequant.cpp:268-301, :359-402, :739-780), compiled
  from its sources into oracle/_ref/libvbref.so by oracle/build.py.
* Q8_0 dequant: the reference's numpy loader ``_dequant_q8_0`` (vibeblade/loader.py:129-133),
  imported by file path (the GGUF fp16-scale block the reference's CUDA kernel also
  uses).  The C++ CPU reading (float32 scale, cpp/src/dequant.cpp:99-112) of the same
  bytes is stored too, as the record of that defect.
* Q6_K known answers: the uniform-pattern cases of the reference's tests/test_kquants.py:
  134-176 (ql=0xFF,qh=0xFF -> 31; zeros -> -32; qh=0x55 -> -16 with d=1, scale=1).

The weights are this library's own quantizer output (the reference ships no k-quant
quantizer) plus hand-built edge-case blocks: d = 0, subnormal d / dmin, negative d and
dmin, all-0xFF bytes, and random bytes with finite fp16 scales.
"""
from __future__ import annotations

import importlib.util
import os
import struct
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.dont_write_bytecode = True  # never write into the read-only reference checkout

from oracle.build import ref_root  # noqa: E402
from oracle.oracle import load_ref  # noqa: E402
from vibeblade_b200 import formats as F  # noqa: E402
from vibeblade_b200.quantize import quantize  # noqa: E402

REF = ref_root()
K, N, B = 32, 512, 4


def _loader_q8_0():
    spec = importlib.util.spec_from_file_location("_vb_ref_loader", REF / "vibeblade" / "loader.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod._dequant_q8_0


def _f16(v: float) -> bytes:
    return struct.pack("<e", v)


def edge_rows(qtype: int, rng: np.random.Generator, n: int) -> np.ndarray:
    """Rows of hand-made blocks covering the scale edge cases."""
    bb, bv = F.BLOCK_BYTES[qtype], F.BLOCK_VALUES[qtype]
    nb = n // bv
    rows = []
    # scale field offsets per type: list of (offset) of fp16 scales
    scale_offs = {F.GGML_TYPE_Q4_K: [0, 2], F.GGML_TYPE_Q6_K: [208], F.GGML_TYPE_Q8_0: [0]}[qtype]
    specials = [0.0, 5.96e-08, 3.0e-05, 6.1e-05, -0.0123, 1.0, -2.5, 0.001, 65504.0, -6.0e-07]
    for variant in range(8):
        blocks = bytearray(rng.integers(0, 256, size=nb * bb, dtype=np.uint8).tobytes())
        for b in range(nb):
            base = b * bb
            if variant == 0:           # all 0xFF body, finite scales
                for i in range(bb):
                    blocks[base + i] = 0xFF
            if variant == 1:           # all-zero body
                for i in range(bb):
                    blocks[base + i] = 0
            for so in scale_offs:
                v = specials[(b + variant * 3 + so) % len(specials)]
                blocks[base + so: base + so + 2] = _f16(v)
        rows.append(np.frombuffer(bytes(blocks), np.uint8))
    return np.stack(rows)


def q6k_known_answers() -> dict:
    out = {}
    for name, ql, qh, want in (("max", 0xFF, 0xFF, 31.0), ("min", 0x00, 0x00, -32.0),
                               ("mid", 0x00, 0x55, -16.0)):
        blk = bytearray(210)
        blk[208:210] = _f16(1.0)
        for i in range(192, 208):
            blk[i] = 1
        for i in range(128):
            blk[i] = ql
        for i in range(128, 192):
            blk[i] = qh
        out[f"q6k_ka_{name}_bytes"] = np.frombuffer(bytes(blk), np.uint8)
        out[f"q6k_ka_{name}_want"] = np.full(256, want, np.float32)
    return out


def main() -> None:
    ref = load_ref()
    if ref is None:
        raise SystemExit("reference sources not found; set VB_REF")
    deq_q8 = _loader_q8_0()
    for qtype in (F.GGML_TYPE_Q4_K, F.GGML_TYPE_Q6_K, F.GGML_TYPE_Q8_0):
        name = F.TYPE_NAMES[qtype].lower()
        rng = np.random.default_rng(1000 + qtype)
        wq = quantize(rng.normal(0.0, 0.02, size=(K, N)).astype(np.float32), qtype).numpy()
        we = edge_rows(qtype, rng, N)
        w = np.concatenate([wq, we], axis=0)
        rows = w.shape[0]
        x = rng.normal(0.0, 1.0, size=(B, rows)).astype(np.float32)
        rec = {"w": w, "x": x, "K": np.int64(rows), "N": np.int64(N), "type": np.int64(qtype)}
        if qtype == F.GGML_TYPE_Q8_0:
            bb = 34
            deq = np.stack([np.concatenate([deq_q8(bytes(w[r, j * bb:(j + 1) * bb]))
                                            for j in range(N // 32)]) for r in range(rows)])
            rec["deq"] = deq.astype(np.float32)
            rec["deq_cpp_f32scale"] = np.stack([ref.dequantize_row(w[r], N, qtype) for r in range(rows)])
            # no reference gemv for the fp16-scale block: exact sum of the loader's values
            rec["gemv_f64"] = (x.astype(np.float64) @ deq.astype(np.float64))
        else:
            rec["deq"] = np.stack([ref.dequantize_row(w[r], N, qtype) for r in range(rows)])
            rec["gemv"] = ref.gemv_dequant(x, w, rows, N, qtype)
            rec["gemv_f64"] = x.astype(np.float64) @ rec["deq"].astype(np.float64)
            # a ragged single row (n not a block multiple)
            n_rag = 200
            rec["ragged_n"] = np.int64(n_rag)
            rec["ragged_deq"] = ref.dequantize_row(w[0], n_rag, qtype)
        np.savez_compressed(HERE / f"{name}.npz", **rec)
        print(name, {k: v.shape for k, v in rec.items()})
    np.savez_compressed(HERE / "q6k_known_answers.npz", **q6k_known_answers())


if __name__ == "__main__":
    main()
