"""Golden vectors for the reference dispatcher's other block types (Q4_0, Q4_1, Q5_0,
Q5_1, Q2_K, Q3_K, Q5_K, Q8_K) from the reference itself: its own ``dequantize_row`` and
``gemv_dequant`` (cpp/src/dequant.cpp:23-245, :317-354, :407-425, :739-780), compiled from
its sources into oracle/_ref/libvbref.so by oracle/build.py.

Run where the reference checkout is mounted (``$VB_REF`` names it):

    python tests/golden/make_blocks_golden.py

Writes tests/golden/blocks.npz: per type ``<name>_w`` (16 rows of 512 values: 8 rows of
random codes with N(0, 0.01) scales, 8 edge rows), ``<name>_deq``, ``<name>_x`` [3, 16],
``<name>_gemv`` (the reference's sequential fp32 sums), ``<name>_ragged_deq`` (the first
row dequantized with n = 200) and ``<name>_random_w`` / ``<name>_random_deq`` (rows of
unconstrained random bytes: inf and NaN scales included).
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(HERE.parent))
sys.dont_write_bytecode = True  # never write into the read-only reference checkout

from block_fill import BLOCK_BYTES, BLOCK_VALUES, TYPES, edge_blocks, random_blocks  # noqa: E402
from oracle.oracle import load_ref  # noqa: E402
from vibeblade_b200 import formats as F  # noqa: E402

K, N, B, N_RAGGED = 16, 512, 3, 200


def main() -> None:
    ref = load_ref()
    if ref is None:
        raise SystemExit("reference sources not found; set VB_REF")
    rec = {"K": np.int64(K), "N": np.int64(N), "ragged_n": np.int64(N_RAGGED)}
    for qtype in TYPES:
        name = F.TYPE_NAMES[qtype].lower()
        rng = np.random.default_rng(2000 + qtype)
        w = np.concatenate([random_blocks(qtype, K // 2, N, rng), edge_blocks(qtype, K // 2, N, rng)])
        x = rng.normal(0.0, 1.0, size=(B, K)).astype(np.float32)
        rec[f"{name}_w"] = w
        rec[f"{name}_deq"] = np.stack([ref.dequantize_row(w[r], N, qtype) for r in range(K)])
        rec[f"{name}_x"] = x
        rec[f"{name}_gemv"] = ref.gemv_dequant(x, w, K, N, qtype)
        rec[f"{name}_ragged_deq"] = ref.dequantize_row(w[0], N_RAGGED, qtype)
        wr = rng.integers(0, 256, size=(4, N // BLOCK_VALUES[qtype] * BLOCK_BYTES[qtype]), dtype=np.uint8)
        rec[f"{name}_random_w"] = wr
        rec[f"{name}_random_deq"] = np.stack([ref.dequantize_row(wr[r], N, qtype) for r in range(4)])
    np.savez_compressed(HERE / "blocks.npz", **rec)
    print({k: v.shape for k, v in rec.items()})


if __name__ == "__main__":
    main()
