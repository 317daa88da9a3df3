"""Weight bytes for the block types that have no quantizer here (Q4_0, Q4_1, Q5_0, Q5_1,
Q2_K, Q3_K, Q5_K, Q8_K).  The reference ships no quantizer for them either; its
dequantizers are functions of the bytes alone, so random code bytes with the scale fields
overwritten by finite values of a chosen size cover every path a real file takes, and the
edge rows add the scale cases files can hold (zero, fp16 subnormal -- which the
reference's f16_to_f32 doubles -- negative, the largest fp16) and all-0x00 / all-0xFF
bodies.  Used by the tests and by tests/golden/make_blocks_golden.py."""
from __future__ import annotations

import struct

import numpy as np

# (byte offset, struct code) of each scale field in a block: fp16 'e' or fp32 'f'
# (cpp/include/ggml_types.h:82-168)
SCALE_FIELDS = {
    2: [(0, "e")],                # Q4_0: d
    3: [(0, "e"), (2, "e")],      # Q4_1: d, m
    6: [(0, "e")],                # Q5_0: d
    7: [(0, "e"), (2, "e")],      # Q5_1: d, m
    10: [(80, "e"), (82, "e")],   # Q2_K: d, dmin
    11: [(108, "e")],             # Q3_K: d
    13: [(0, "e"), (2, "e")],     # Q5_K: d, dmin
    15: [(0, "f")],               # Q8_K: d (fp32)
}
BLOCK_VALUES = {2: 32, 3: 32, 6: 32, 7: 32, 10: 256, 11: 256, 13: 256, 15: 256}
BLOCK_BYTES = {2: 18, 3: 20, 6: 22, 7: 24, 10: 84, 11: 110, 13: 176, 15: 292}
TYPES = tuple(SCALE_FIELDS)

_SPECIAL = [0.0, 5.96e-08, 3.0e-05, 6.1e-05, -0.0123, 1.0, -2.5, 0.001, 65504.0, -6.0e-07]


def _put(buf: np.ndarray, off: int, code: str, v: float) -> None:
    buf[off:off + struct.calcsize("<" + code)] = np.frombuffer(struct.pack("<" + code, v), np.uint8)


def random_blocks(qtype: int, K: int, N: int, rng: np.random.Generator, std: float = 0.01) -> np.ndarray:
    """K rows of N values: random code bytes, every scale field N(0, std)."""
    bb, bv = BLOCK_BYTES[qtype], BLOCK_VALUES[qtype]
    nb = (N + bv - 1) // bv
    w = rng.integers(0, 256, size=(K, nb * bb), dtype=np.uint8)
    blocks = w.reshape(K, nb, bb)
    for off, code in SCALE_FIELDS[qtype]:
        vals = rng.normal(0.0, std, size=(K, nb)).astype(np.float16 if code == "e" else np.float32)
        width = vals.itemsize
        blocks[:, :, off:off + width] = vals.reshape(K, nb, 1).view(np.uint8).reshape(K, nb, width)
    return w


def edge_blocks(qtype: int, K: int, N: int, rng: np.random.Generator) -> np.ndarray:
    """K rows cycling through the edge cases: all-0xFF and all-zero bodies, special scales."""
    bb, bv = BLOCK_BYTES[qtype], BLOCK_VALUES[qtype]
    nb = (N + bv - 1) // bv
    w = rng.integers(0, 256, size=(K, nb * bb), dtype=np.uint8)
    for r in range(K):
        if r % 4 == 0:
            w[r] = 0xFF
        elif r % 4 == 1:
            w[r] = 0
        for b in range(nb):
            for j, (off, code) in enumerate(SCALE_FIELDS[qtype]):
                _put(w[r], b * bb + off, code, _SPECIAL[(3 * r + b + 5 * j) % len(_SPECIAL)])
    return w
