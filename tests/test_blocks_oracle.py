"""The reference dispatcher's other block types -- Q4_0, Q4_1, Q5_0, Q5_1, Q2_K, Q3_K,
Q5_K, Q8_K (cpp/src/dequant.cpp:23-245, :317-354, :407-425) -- in the CPU oracle, pinned
bit for bit to the reference itself: the committed golden vectors its compiled C++ wrote
(tests/golden/make_blocks_golden.py) and, where the compiled reference is present, fresh
random rows, ragged lengths included."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from block_fill import BLOCK_BYTES, BLOCK_VALUES, TYPES, edge_blocks, random_blocks
from conftest import bits_equal, load_golden
from vibeblade_b200 import formats as F

NAMES = [F.TYPE_NAMES[t].lower() for t in TYPES]


@pytest.fixture(scope="module")
def golden():
    return load_golden("blocks")


@pytest.mark.parametrize("name", NAMES)
def test_oracle_matches_reference_golden(oracle, golden, name):
    t = F.NAME_TO_TYPE[name.upper()]
    K, N = int(golden["K"]), int(golden["N"])
    w = golden[f"{name}_w"]
    assert bits_equal(oracle.dequantize(w, K, N, t), golden[f"{name}_deq"])
    # the reference's sequential fp32 gemv_dequant, bit for bit
    assert bits_equal(oracle.gemv_dequant(golden[f"{name}_x"], w, K, N, t), golden[f"{name}_gemv"])
    n = int(golden["ragged_n"])
    assert bits_equal(oracle.dequantize_row(w[0], n, t), golden[f"{name}_ragged_deq"])
    wr = golden[f"{name}_random_w"]  # unconstrained bytes: inf / NaN scales
    assert bits_equal(oracle.dequantize(wr, wr.shape[0], N, t), golden[f"{name}_random_deq"])


@pytest.mark.parametrize("qtype", TYPES)
def test_oracle_vs_compiled_reference_random(oracle, reflib, qtype):
    rng = np.random.default_rng(300 + qtype)
    bv = BLOCK_VALUES[qtype]
    N = 3 * bv if bv == 256 else 7 * bv
    K = 12
    for w in (random_blocks(qtype, K, N, rng, std=0.02), random_blocks(qtype, K, N, rng, std=3e-5),
              edge_blocks(qtype, K, N, rng)):
        ref = np.stack([reflib.dequantize_row(w[r], N, qtype) for r in range(K)])
        assert bits_equal(oracle.dequantize(w, K, N, qtype), ref)
        x = rng.normal(0, 1, (2, K)).astype(np.float32)
        assert bits_equal(oracle.gemv_dequant(x, w, K, N, qtype), reflib.gemv_dequant(x, w, K, N, qtype))
    # ragged single rows: inside a block, one past a block, one short of one
    for n in (1, 7, 31, 33, bv - 1, bv + 1, N - 5):
        row = random_blocks(qtype, 1, N, rng)[0]
        assert bits_equal(oracle.dequantize_row(row, n, qtype), reflib.dequantize_row(row, n, qtype)), n


def test_q8_1_is_unsupported_like_the_reference(oracle):
    """Q8_1 (type 9) is in the reference's enum but not in its dispatcher, which throws
    "Unsupported dequant type" (cpp/src/dequant.cpp:423)."""
    with pytest.raises(RuntimeError, match="Unsupported dequant type"):
        oracle.dequantize_row(np.zeros(40, np.uint8), 32, 9)
    with pytest.raises(RuntimeError, match="Unsupported dequant type"):
        F.parse_type(9)


def test_block_tables_agree():
    for t in TYPES:
        assert F.BLOCK_VALUES[t] == BLOCK_VALUES[t] and F.BLOCK_BYTES[t] == BLOCK_BYTES[t]
        assert F.parse_type(F.TYPE_NAMES[t]) == t


def test_random_block_weights(oracle):
    """The library's synthetic weights for the types without a quantizer (the bench's
    `other_types` object): the reference's block sizes, finite values of the chosen scale,
    and a refusal for the types that have a quantizer."""
    from vibeblade_b200.quantize import random_block_weights
    for t in TYPES:
        w = random_block_weights(8, 512, t, seed=1, std=1e-3)
        assert w.dtype == torch.uint8 and tuple(w.shape) == (8, F.row_bytes(t, 512))
        v = oracle.dequantize(w.numpy(), 8, 512, t)
        assert np.isfinite(v).all() and 0 < np.abs(v).max() < 100  # Q8_K: d * int8 scale * int8 code
    with pytest.raises(ValueError):
        random_block_weights(8, 512, F.GGML_TYPE_Q4_K)
