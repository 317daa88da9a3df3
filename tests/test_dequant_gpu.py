"""Device dequantization vs the reference, bit-exact (fp32) and round-to-nearest-even (bf16).

Inputs: the committed golden vectors (reference C++ / reference numpy loader outputs),
the oracle on seeded quantized matrices, and edge-case blocks (zero, subnormal, negative
scales; all-0xFF and all-zero bodies; random bytes)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import vibeblade_b200 as vb
from conftest import bits_equal, load_golden
from vibeblade_b200 import formats as F
from vibeblade_b200.quantize import quantize, synthetic_weights

pytestmark = pytest.mark.gpu

TYPES = [F.GGML_TYPE_Q4_K, F.GGML_TYPE_Q6_K, F.GGML_TYPE_Q8_0]


def bf16_rne(a: np.ndarray) -> np.ndarray:
    t = torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16)
    return t.float().numpy()


@pytest.mark.parametrize("name", ["q4_k", "q6_k", "q8_0"])
def test_dequant_golden_bitexact(cuda, name):
    g = load_golden(name)
    K, N, t = int(g["K"]), int(g["N"]), int(g["type"])
    w = torch.from_numpy(g["w"]).to(cuda)
    got = vb.dequantize(w, K, N, t).cpu().numpy()
    assert bits_equal(got, g["deq"])
    gb = vb.dequantize(w, K, N, t, dtype=torch.bfloat16).float().cpu().numpy()
    assert bits_equal(gb, bf16_rne(g["deq"]))


@pytest.mark.parametrize("name", ["q4_k", "q6_k"])
def test_dequantize_row_ragged(cuda, name):
    g = load_golden(name)
    n = int(g["ragged_n"])
    row = torch.from_numpy(g["w"][0].copy()).to(cuda)
    got = vb.dequantize_row(row, None, n, int(g["type"])).cpu().numpy()
    assert got.shape == (n,)
    assert bits_equal(got, g["ragged_deq"])


@pytest.mark.parametrize("case", ["max", "min", "mid"])
def test_q6k_known_answers(cuda, case):
    g = load_golden("q6k_known_answers")
    row = torch.from_numpy(g[f"q6k_ka_{case}_bytes"]).to(cuda)
    got = vb.dequantize_row(row, None, 256, F.GGML_TYPE_Q6_K).cpu().numpy()
    assert np.array_equal(got, g[f"q6k_ka_{case}_want"])


@pytest.mark.parametrize("qtype", TYPES)
@pytest.mark.parametrize("shape", [(1, 256), (3, 512), (17, 2048), (64, 4096)])
def test_dequant_random_vs_oracle(cuda, oracle, qtype, shape):
    K, N = shape
    rng = np.random.default_rng(K * 7 + N + qtype)
    w = quantize(rng.normal(0, 0.02, (K, N)).astype(np.float32), qtype).numpy()
    ref = oracle.dequantize(w, K, N, qtype)
    wd = torch.from_numpy(w).to(cuda)
    assert bits_equal(vb.dequantize(wd, K, N, qtype).cpu().numpy(), ref)
    assert bits_equal(vb.dequantize(wd, K, N, qtype, dtype=torch.bfloat16).float().cpu().numpy(),
                      bf16_rne(ref))


@pytest.mark.parametrize("qtype", TYPES)
def test_dequant_random_bytes(cuda, oracle, qtype):
    """Arbitrary bytes, scales included (inf/NaN scales give NaN outputs on both sides)."""
    K, N = 8, 1024
    rng = np.random.default_rng(5 + qtype)
    w = rng.integers(0, 256, size=(K, F.row_bytes(qtype, N)), dtype=np.uint8)
    ref = oracle.dequantize(w, K, N, qtype)
    got = vb.dequantize(torch.from_numpy(w).to(cuda), K, N, qtype).cpu().numpy()
    assert bits_equal(got, ref)


@pytest.mark.parametrize("qtype", TYPES)
def test_dequant_full_size_rows_sampled(cuda, oracle, qtype):
    """A BASELINE-size matrix (4096 x 14336) dequantized on the device; sampled rows
    compared bit-exactly with the oracle."""
    K, N = 4096, 14336
    wd = synthetic_weights(K, N, qtype, seed=0, device=cuda)
    out = vb.dequantize(wd, K, N, qtype)
    rows = [0, 1, 777, 2048, 4095]
    wh = wd[rows].cpu().numpy()
    ref = oracle.dequantize(wh, len(rows), N, qtype)
    assert bits_equal(out[rows].cpu().numpy(), ref)
    assert torch.isfinite(out).all()


def test_dequant_empty_is_noop(cuda):
    w = torch.zeros(144, dtype=torch.uint8, device=cuda)
    out = vb.dequantize(w, 0, 256, F.GGML_TYPE_Q4_K)
    assert out.shape == (0, 256)


@pytest.mark.parametrize("qtype", [F.GGML_TYPE_F32, F.GGML_TYPE_F16, F.GGML_TYPE_BF16])
@pytest.mark.parametrize("K,N", [(1, 65536), (3, 1000), (17, 8)])
def test_dequant_unquantized_rows_bitexact(cuda, oracle, qtype, K, N):
    """F32 / F16 / BF16 weights: every 16-bit pattern (F16 subnormals doubled as the
    reference's f16_to_f32 does), widths that end inside a lane's 8 values, and a single
    ragged row; bit-exact against the oracle (pinned to the compiled reference)."""
    rng = np.random.default_rng(K * 7 + N + qtype)
    eb = F.BLOCK_BYTES[qtype]
    if qtype == F.GGML_TYPE_F32:
        w = rng.normal(0, 1, K * N).astype(np.float32).view(np.uint8)
    else:
        w = rng.integers(0, 65536, K * N, dtype=np.uint16)
        w[:min(w.size, 65536)] = np.arange(min(w.size, 65536), dtype=np.uint16)
        w = w.view(np.uint8)
    want = oracle.dequantize(w, K, N, qtype)
    got = vb.dequantize(torch.from_numpy(w).to(cuda), K, N, qtype).cpu().numpy()
    assert bits_equal(got, want)
    gb = vb.dequantize(torch.from_numpy(w).to(cuda), K, N, qtype, dtype=torch.bfloat16).float().cpu().numpy()
    assert bits_equal(gb, bf16_rne(want))
    # one ragged row
    n1 = N - 3 if N > 3 else N
    row = vb.dequantize_row(torch.from_numpy(w[:N * eb].copy()).to(cuda), None, n1, qtype).cpu().numpy()
    assert bits_equal(row, want[0, :n1])
