"""The batch 5..16 Q4_K GEMV on the fp16 tensor cores (vbq_gemv_half.cu) through its
scale paths: a per-CTA, per-batch-row power-of-two scale set from the first stage, set
again when a later stage outgrows it (the sums so far multiplied by the exact ratio) or
when the first stage held only zeros, and non-finite activations marking their row.
Batches 2..4 run the same cases through the integer kernel (vbq_gemv_mma.cu).

Reference: the reference's gemv_dequant (cpp/src/dequant.cpp:739-780), here its oracle
restatement (sequential fp32) and an fp64 product of the bit-exact dequantization, with
the max-norm 1e-3 bar and the per-column bar of test_gemv_gpu.py."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import vibeblade_b200 as vb
from vibeblade_b200 import formats as F
from vibeblade_b200.quantize import quantize, synthetic_weights

pytestmark = pytest.mark.gpu

Q4 = F.GGML_TYPE_Q4_K
TOL = 1e-3


def _check(y, ref, what):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    mx = np.abs(ref).max(axis=1, keepdims=True)
    err = np.abs(y - ref)
    assert (err / mx).max() <= TOL, f"{what}: max-norm {(err / mx).max():.3g}"
    big = np.abs(ref) >= 1e-2 * mx
    rel = err[big] / np.abs(ref[big])
    assert rel.max() <= TOL, f"{what}: per-column {rel.max():.3g}"


def _ref64(cuda, x, w, K, N):
    deq = vb.dequantize(w, K, N, Q4).double()
    return (torch.from_numpy(x).to(cuda).double() @ deq).cpu().numpy()


@pytest.mark.parametrize("batch", [2, 3, 4, 7, 8, 12, 16])
@pytest.mark.parametrize("K,N", [(4096, 1024), (1000, 512), (14336, 512)])
def test_half_scale_paths(cuda, oracle, batch, K, N):
    """Rows whose first 64-row stage is all zeros (scale unset, set by a later stage),
    rows that grow 10^4-fold half-way down (the scale set again mid-matrix), ordinary
    rows; every K-split of the tile meets these at its own first stage."""
    rng = np.random.default_rng(K + N + batch)
    w = synthetic_weights(K, N, Q4, seed=K + N, device=cuda)
    x = rng.normal(0, 1, (batch, K)).astype(np.float32)
    x[0, : min(K, 700)] = 0.0
    if batch > 1:
        x[1, K // 2:] *= 1e4
    if batch > 2:
        x[2, : K // 3] *= 1e-3
    y = vb.gemv_dequant(torch.from_numpy(x).to(cuda), w, None, K, N, Q4).cpu().numpy()
    assert vb.device_status() == 0
    _check(y, _ref64(cuda, x, w, K, N), "fp64")
    _check(y, oracle.gemv_dequant(x, w.cpu().numpy(), K, N, Q4), "oracle")


@pytest.mark.parametrize("batch", [4, 16])
def test_half_all_zero_row(cuda, batch):
    """A batch row of zeros never sets its scale; its outputs are exact zeros."""
    K, N = 2048, 512
    w = synthetic_weights(K, N, Q4, seed=5, device=cuda)
    x = torch.randn(batch, K, device=cuda)
    x[1].zero_()
    y = vb.gemv_dequant(x, w, None, K, N, Q4)
    assert torch.equal(y[1], torch.zeros(N, device=cuda))
    assert torch.isfinite(y).all()


@pytest.mark.parametrize("bad", [float("nan"), float("inf")])
@pytest.mark.parametrize("batch", [3, 8, 16])
def test_half_nonfinite_marks_its_row(cuda, oracle, bad, batch):
    """A non-finite activation makes every output of its batch row NaN (the reference's
    fp32 sum is NaN or +-inf there); the other rows are unaffected."""
    K, N = 1024, 512
    rng = np.random.default_rng(batch)
    wn = quantize(rng.normal(0, 0.02, (K, N)).astype(np.float32), Q4).numpy()
    x = rng.normal(0, 1, (batch, K)).astype(np.float32)
    x[1, 777] = bad
    y = vb.gemv_dequant(torch.from_numpy(x).to(cuda), torch.from_numpy(wn).to(cuda), None, K, N,
                        Q4).cpu().numpy()
    assert np.isnan(y[1]).all()
    ok = [b for b in range(batch) if b != 1]
    ref = oracle.gemv_dequant(x[ok], wn, K, N, Q4)
    _check(y[ok], ref, "oracle")


@pytest.mark.parametrize("batch", [2, 5, 8, 16])
def test_half_swiglu_input(cuda, oracle, batch):
    """The down projection reading silu(gate) * up from a [batch, 2K] gate | up buffer."""
    K, N = 2048, 1024
    rng = np.random.default_rng(100 + batch)
    w = synthetic_weights(K, N, Q4, seed=77, device=cuda)
    gu = rng.normal(0, 2, (batch, 2 * K)).astype(np.float32)
    g, u = gu[:, :K].astype(np.float64), gu[:, K:].astype(np.float64)
    h = (g / (1.0 + np.exp(-g)) * u).astype(np.float32)
    y = vb.gemv_fused(torch.from_numpy(gu).to(cuda), w, None, K, N, Q4, swiglu_input=True)
    assert vb.device_status() == 0
    _check(y.cpu().numpy(), _ref64(cuda, h, w, K, N), "fp64")


@pytest.mark.parametrize("batch", [4, 16])
def test_half_deterministic_and_epilogue(cuda, batch):
    """Repeated calls are bit-identical; bias and residual add in the epilogue."""
    K, N = 4096, 2048
    w = synthetic_weights(K, N, Q4, seed=9, device=cuda)
    x = torch.randn(batch, K, device=cuda)
    bias = torch.randn(N, device=cuda)
    res = torch.randn(batch, N, device=cuda)
    y0 = vb.gemv_dequant(x, w, None, K, N, Q4)
    for _ in range(3):
        assert torch.equal(vb.gemv_dequant(x, w, None, K, N, Q4), y0)
    yf = vb.gemv_fused(x, w, None, K, N, Q4, bias=bias, residual=res)
    torch.testing.assert_close(yf, y0 + bias + res, rtol=0, atol=1e-5)
    assert vb.device_status() == 0
