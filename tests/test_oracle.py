"""The CPU oracle pinned against the reference: golden vectors made by the reference's own
compiled C++ and numpy loader, the reference's Q6_K known answers, and (where the
compiled reference library is present) randomized bit-exact comparisons."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import bits_equal, load_golden, max_rel
from vibeblade_b200 import formats as F
from vibeblade_b200.quantize import quantize


@pytest.mark.parametrize("name", ["q4_k", "q6_k", "q8_0"])
def test_oracle_dequant_matches_golden(oracle, name):
    g = load_golden(name)
    K, N, t = int(g["K"]), int(g["N"]), int(g["type"])
    got = oracle.dequantize(g["w"], K, N, t)
    assert bits_equal(got, g["deq"])


@pytest.mark.parametrize("name", ["q4_k", "q6_k"])
def test_oracle_gemv_matches_reference_bitwise(oracle, name):
    g = load_golden(name)
    K, N, t = int(g["K"]), int(g["N"]), int(g["type"])
    got = oracle.gemv_dequant(g["x"], g["w"], K, N, t)
    # same sequential fp32 accumulation as cpp/src/dequant.cpp:772-779
    assert bits_equal(got, g["gemv"])


def test_oracle_q8_0_gemv_close_to_exact_sum(oracle):
    g = load_golden("q8_0")
    K, N, t = int(g["K"]), int(g["N"]), int(g["type"])
    got = oracle.gemv_dequant(g["x"], g["w"], K, N, t)
    fin = np.isfinite(g["gemv_f64"]).all(axis=0)
    assert max_rel(got[:, fin], g["gemv_f64"][:, fin]) < 1e-5


@pytest.mark.parametrize("name", ["q4_k", "q6_k"])
def test_oracle_ragged_row(oracle, name):
    g = load_golden(name)
    n = int(g["ragged_n"])
    got = oracle.dequantize_row(g["w"][0], n, int(g["type"]))
    assert bits_equal(got, g["ragged_deq"])


@pytest.mark.parametrize("case", ["max", "min", "mid"])
def test_oracle_q6k_known_answers(oracle, case):
    """tests/test_kquants.py:134-176 of the reference: uniform byte patterns."""
    g = load_golden("q6k_known_answers")
    got = oracle.dequantize_row(g[f"q6k_ka_{case}_bytes"], 256, F.GGML_TYPE_Q6_K)
    assert np.array_equal(got, g[f"q6k_ka_{case}_want"])


def test_q8_0_cpp_reader_is_a_documented_reference_defect(oracle):
    """Documented reference defect: the C++ CPU dequantize_row_q8_0
    (cpp/src/dequant.cpp:99-112) reads a float32 scale from bytes 0-3 of each 34-byte
    block, where GGUF (and the reference's own CUDA kernel and numpy loader) store an
    fp16 scale at bytes 0-1.  The restatement of that reading reproduces the reference's
    output, and it differs from the fp16-scale values this library computes."""
    g = load_golden("q8_0")
    K, N = int(g["K"]), int(g["N"])
    def padded(row):  # the C++ reader runs 2 bytes past the row; the golden padded zeros
        buf = np.zeros(row.size + 64, np.uint8)
        buf[:row.size] = row
        return buf

    cpp = np.stack([oracle.dequantize_q8_0_f32scale(padded(g["w"][r]), N) for r in range(K)])
    assert bits_equal(cpp, g["deq_cpp_f32scale"])
    assert not bits_equal(cpp, g["deq"])


def test_f16_conversion_follows_reference(oracle):
    """f16_to_f32 (cpp/src/fp16_compat.cpp:13-35): exact for normals, inf, NaN payloads;
    subnormals come out doubled.  The IEEE variant is exact everywhere."""
    h = np.arange(65536, dtype=np.uint16)
    ieee = h.view(np.float16).astype(np.float32)
    ref = np.array([oracle.f16_to_f32(int(v)) for v in h], np.float32)
    ie = np.array([oracle.f16_to_f32_ieee(int(v)) for v in h], np.float32)
    sub = ((h & 0x7C00) == 0) & ((h & 0x3FF) != 0)
    assert bits_equal(ie, ieee)
    assert bits_equal(ref[~sub], ieee[~sub])
    assert np.array_equal(ref[sub], ieee[sub] * 2)


@pytest.mark.parametrize("qtype", [F.GGML_TYPE_Q4_K, F.GGML_TYPE_Q6_K])
@pytest.mark.parametrize("std", [0.02, 1.0, 3e-5])
def test_oracle_vs_compiled_reference_random(oracle, reflib, qtype, std):
    rng = np.random.default_rng(int(std * 1e6) + qtype)
    K, N = 24, 768
    w = quantize(rng.normal(0, std, (K, N)).astype(np.float32), qtype).numpy()
    # random bytes with finite scales too
    wr = rng.integers(0, 256, size=w.shape, dtype=np.uint8)
    for r in range(K):
        for b in range(N // 256):
            base = b * F.BLOCK_BYTES[qtype]
            for off in ([0, 2] if qtype == F.GGML_TYPE_Q4_K else [208]):
                wr[r, base + off: base + off + 2] = np.frombuffer(
                    np.float16(rng.normal(0, 0.01)).tobytes(), np.uint8)
    for wm in (w, wr):
        ref = np.stack([reflib.dequantize_row(wm[r], N, qtype) for r in range(K)])
        assert bits_equal(oracle.dequantize(wm, K, N, qtype), ref)
        x = rng.normal(0, 1, (2, K)).astype(np.float32)
        assert bits_equal(oracle.gemv_dequant(x, wm, K, N, qtype), reflib.gemv_dequant(x, wm, K, N, qtype))


@pytest.mark.parametrize("qtype", [F.GGML_TYPE_F32, F.GGML_TYPE_F16, F.GGML_TYPE_BF16])
def test_oracle_unquantized_rows_vs_compiled_reference(oracle, reflib, qtype):
    """F32 / F16 / BF16 rows (the reference's dequantize_row, cpp/src/dequant.cpp:407-411):
    every 16-bit pattern once (F16 subnormals double, NaN and inf pass through), and a GEMV
    over random weights, bit for bit against the compiled reference."""
    rng = np.random.default_rng(qtype + 5)
    if qtype == F.GGML_TYPE_F32:
        row = rng.normal(0, 1, 4096).astype(np.float32).view(np.uint8)
        n = 4096
    else:
        row = np.arange(65536, dtype=np.uint16).view(np.uint8)
        n = 65536
    assert bits_equal(oracle.dequantize_row(row, n, qtype), reflib.dequantize_row(row, n, qtype))
    K, N = 64, 40  # a width that is no multiple of any block but the unquantized one
    vals = rng.normal(0, 0.05, (K, N)).astype(np.float32)
    w = {F.GGML_TYPE_F32: vals, F.GGML_TYPE_F16: vals.astype(np.float16),
         F.GGML_TYPE_BF16: (vals.view(np.uint32) >> 16).astype(np.uint16)}[qtype]
    x = rng.normal(0, 1, (3, K)).astype(np.float32)
    assert bits_equal(oracle.gemv_dequant(x, w, K, N, qtype), reflib.gemv_dequant(x, w, K, N, qtype))
