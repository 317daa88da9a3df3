"""The batch 1-4 Q6_K GEMV on the integer tensor cores (vbq_gemv_q6.cu) through its own
paths: the per-warp, per-batch-row power-of-two scale of v = x * d * sc (set from the first
stage, set again
when a stage outgrows it or falls 16x below it, or when the first stage held only
zeros), the -32 offset taken off through the sums of v, codes and scales at their
extremes, rows whose 16-byte copy window reaches the end of the matrix, the cluster
split-K, and non-finite activations.

Reference: the reference's gemv_dequant (cpp/src/dequant.cpp:739-780) over its Q6_K
dequantization (:359-402), here the oracle restatement (sequential fp32) and an fp64
product of the bit-exact device dequantization, with the max-norm 1e-3 bar and the
per-column bar of test_gemv_gpu.py."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import vibeblade_b200 as vb
from vibeblade_b200 import formats as F
from vibeblade_b200.quantize import quantize, synthetic_weights

pytestmark = pytest.mark.gpu

Q6 = F.GGML_TYPE_Q6_K
TOL = 1e-3


def _check(y, ref, what):
    y = np.asarray(y, np.float64).reshape(-1)
    ref = np.asarray(ref, np.float64).reshape(-1)
    mx = np.abs(ref).max()
    err = np.abs(y - ref)
    assert (err / mx).max() <= TOL, f"{what}: max-norm {(err / mx).max():.3g}"
    big = np.abs(ref) >= 1e-2 * mx
    rel = err[big] / np.abs(ref[big])
    assert rel.max() <= TOL, f"{what}: per-column {rel.max():.3g}"


def _ref64(cuda, x, w, K, N):
    deq = vb.dequantize(w, K, N, Q6).double()
    return (torch.as_tensor(x, device=cuda).double().reshape(-1, K) @ deq).cpu().numpy()


def _check_rows(y, ref, what):
    """_check per batch row; a row whose reference is all zeros (x row of zeros) must come
    out exactly zero."""
    ref = np.asarray(ref, np.float64)
    ref = ref.reshape(-1, ref.shape[-1])
    y = np.asarray(y, np.float64).reshape(ref.shape)
    for b in range(ref.shape[0]):
        if not np.abs(ref[b]).max() > 0:
            assert np.array_equal(y[b], np.zeros_like(y[b])), f"{what} row {b}: not all zeros"
        else:
            _check(y[b], ref[b], f"{what} row {b}")


@pytest.mark.parametrize("batch", [1, 2, 3, 4])
@pytest.mark.parametrize("K,N", [(4096, 1024), (1000, 512), (14336, 4096), (4096, 12288)])
def test_q6_scale_paths(cuda, oracle, K, N, batch):
    """Rows whose first stages are all zeros (scale unset, set by a later stage), rows that
    grow 10^4-fold half-way down (set again mid-matrix) and rows 10^-3 smaller (the scale
    comes back down); each K-split of a tile meets them at its own first stage.  At batch 2
    the second row has a different profile, so the two rows' scales move independently."""
    rng = np.random.default_rng(K + N)
    w = synthetic_weights(K, N, Q6, seed=K + N, device=cuda)
    x = rng.normal(0, 1, (batch, K)).astype(np.float32)
    x[0, : min(K, 700)] = 0.0
    x[0, K // 2:] *= 1e4
    x[0, K // 3: K // 2] *= 1e-3
    if batch > 1:
        x[1, : K // 4] *= 1e3
        x[1, K - min(K, 300):] = 0.0
    if batch > 3:
        x[3] = 0.0  # a batch row of zeros never sets its scale
    y = vb.gemv_dequant(torch.from_numpy(x).to(cuda), w, None, K, N, Q6).cpu().numpy()
    assert vb.device_status() == 0
    _check_rows(y, _ref64(cuda, x, w, K, N), "fp64")
    if K * N <= 4096 * 4096:
        _check_rows(y, oracle.gemv_dequant(x, w.cpu().numpy(), K, N, Q6), "oracle")


def _blocks(K, N, rng, ql=None, qh=None, sc=None, d=None):
    """Raw Q6_K rows [K, N / 256 * 210] with the given fields (random where None)."""
    nb = N // 256
    b = rng.integers(0, 256, (K, nb, 210), dtype=np.uint8)
    if ql is not None:
        b[:, :, :128] = ql
    if qh is not None:
        b[:, :, 128:192] = qh
    if sc is not None:
        b[:, :, 192:208] = np.uint8(sc & 0xff)
    dd = np.full((K, nb), d if d is not None else 0.01, np.float16).view(np.uint8).reshape(K, nb, 2)
    b[:, :, 208:210] = dd
    return b.reshape(K, nb * 210)


@pytest.mark.parametrize("batch", [1, 2, 3, 4])
@pytest.mark.parametrize("ql,qh,sc", [(0xff, 0xff, 127), (0x00, 0x00, -128), (0xff, 0xff, -128),
                                      (0x0f, 0xaa, -1), (None, None, None), (None, None, -128)])
def test_q6_extreme_codes_and_scales(cuda, oracle, ql, qh, sc, batch):
    """Codes at 63 and 0 (q = 31 and -32) and scales at +127 / -128: the u8 codes, the s8
    digits and the int32 centring at the ends of their ranges."""
    K, N = 1000, 768
    rng = np.random.default_rng(7)
    w = _blocks(K, N, rng, ql, qh, sc)
    x = rng.normal(0, 1, (batch, K)).astype(np.float32)
    y = vb.gemv_dequant(torch.from_numpy(x).to(cuda), torch.from_numpy(w).to(cuda), None, K, N,
                        Q6).cpu().numpy()
    assert vb.device_status() == 0
    _check_rows(y, oracle.gemv_dequant(x, w, K, N, Q6), "oracle")


@pytest.mark.parametrize("batch", [1, 2, 3, 4])
@pytest.mark.parametrize("K", [1, 2, 3, 127, 128, 129, 255, 333])
@pytest.mark.parametrize("N", [256, 768, 1280])
def test_q6_matrix_end_windows(cuda, oracle, K, N, batch):
    """Row pitches of 210, 630 and 1050 bytes: the blocks sit at every even offset of their
    16-byte windows, and the block that ends the matrix has its last bytes past the final
    16-byte boundary whenever K * pitch is not a multiple of 16."""
    rng = np.random.default_rng(K * 7 + N)
    w = quantize(rng.normal(0, 0.3, (K, N)).astype(np.float32), Q6).numpy()
    x = rng.normal(0, 1, (batch, K)).astype(np.float32)
    y = vb.gemv_dequant(torch.from_numpy(x).to(cuda), torch.from_numpy(w).to(cuda), None, K, N,
                        Q6).cpu().numpy()
    _check_rows(y, oracle.gemv_dequant(x, w, K, N, Q6), "oracle")


@pytest.mark.parametrize("bad", [float("nan"), float("inf"), float("-inf")])
def test_q6_nonfinite_x(cuda, oracle, bad):
    """A non-finite activation makes every output of its batch row NaN (the reference's fp32
    sum is NaN or +-inf there); at batch 2 and 4 the other rows are unaffected."""
    K, N = 2048, 1024
    w = synthetic_weights(K, N, Q6, seed=3, device=cuda)
    x = torch.randn(K, device=cuda)
    x[1234] = bad
    y = vb.gemv_dequant(x, w, None, K, N, Q6)
    assert torch.isnan(y).all()
    assert vb.device_status() == 0
    for batch, row in ((2, 1), (4, 2)):
        x2 = torch.randn(batch, K, device=cuda)
        x2[row, 777] = bad
        y2 = vb.gemv_dequant(x2, w, None, K, N, Q6)
        assert torch.isnan(y2[row]).all()
        assert vb.device_status() == 0
        ok = [b for b in range(batch) if b != row]
        _check_rows(y2[ok].cpu().numpy(), _ref64(cuda, x2[ok], w, K, N), "fp64")


@pytest.mark.parametrize("batch", [1, 2, 3, 4])
def test_q6_swiglu_input_and_epilogue(cuda, batch):
    """silu(gate) * up read from a [batch, 2K] buffer; bias and residual added in the
    epilogue; repeated calls bit-identical."""
    K, N = 14336, 4096
    w = synthetic_weights(K, N, Q6, seed=11, device=cuda)
    gu = torch.randn(batch, 2 * K, device=cuda) * 2
    h = torch.nn.functional.silu(gu[:, :K].double()) * gu[:, K:].double()
    y = vb.gemv_fused(gu, w, None, K, N, Q6, swiglu_input=True)
    assert vb.device_status() == 0
    ref = (h @ vb.dequantize(w, K, N, Q6).double()).cpu().numpy()
    _check_rows(y.cpu().numpy(), ref, "fp64")
    x = torch.randn(batch, K, device=cuda)
    bias = torch.randn(N, device=cuda)
    res = torch.randn(batch, N, device=cuda)
    y0 = vb.gemv_dequant(x, w, None, K, N, Q6)
    for _ in range(3):
        assert torch.equal(vb.gemv_dequant(x, w, None, K, N, Q6), y0)
    yf = vb.gemv_fused(x, w, None, K, N, Q6, bias=bias, residual=res)
    torch.testing.assert_close(yf, y0 + bias + res, rtol=0, atol=1e-5)


@pytest.mark.parametrize("batch", [1, 2, 3, 4])
@pytest.mark.parametrize("N", [256, 2048, 8192, 37888, 49152, 65536])
def test_q6_split_widths(cuda, N, batch):
    """Tile counts from 1 (the cluster split-K at its widest) through one wave of clusters
    to more tiles than CTA slots (two splits over several waves, or one split filling a
    wave); no scratch is needed at batch 1-4."""
    K = 8192
    assert vb.gemv_scratch_bytes(K, N, Q6, batch) == 0
    w = synthetic_weights(K, N, Q6, seed=N, device=cuda)
    x = torch.randn(batch, K, device=cuda)
    y = vb.gemv_dequant(x, w, None, K, N, Q6)
    assert vb.device_status() == 0
    _check_rows(y.cpu().numpy(), _ref64(cuda, x, w, K, N), "fp64")
