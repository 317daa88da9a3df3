"""tcgen05 quantized-weight GEMM (prefill) vs the reference.

The reference computes prefill as one gemv_dequant per token (cpp/src/fast_model.cpp:
645-660); its exact value is sum_k a[m,k] * deq(W)[k,n] with deq bit-exact to
dequantize_row.  The device path multiplies bf16 activations by bf16-rounded dequantized
weights with fp32 accumulation, so the bar is the north star's 2e-2 max-norm relative
error against an fp64 sum over the bf16-rounded A and the exact dequantized W (oracle)
or, at BASELINE sizes, against fp32 matmul of the bit-exact device dequantization.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import vibeblade_b200 as vb
from conftest import max_rel
from vibeblade_b200 import formats as F
from vibeblade_b200.quantize import quantize, synthetic_weights
from vibeblade_b200.tp import swiglu

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _case(cuda, oracle, qtype, M, K, N, seed, out_dtype=torch.float32):
    rng = np.random.default_rng(seed)
    w = quantize(rng.normal(0, 0.02, (K, N)).astype(np.float32), qtype).numpy()
    a = torch.from_numpy(rng.normal(0, 1, (M, K)).astype(np.float32)).to(torch.bfloat16)
    ref = oracle.gemm_f64(a.float().numpy(), w, M, K, N, qtype)
    c = vb.gemm_dequant(a.to(cuda), torch.from_numpy(w).to(cuda), None, M, K, N, qtype,
                        out_dtype=out_dtype)
    torch.cuda.synchronize()
    assert vb.device_status() == 0
    return c.float().cpu().numpy(), ref


def test_gemm_first_tile(cuda, oracle):
    """One CTA, one K step: the smallest case the pipeline has."""
    c, ref = _case(cuda, oracle, F.GGML_TYPE_Q4_K, 256, 64, 256, 0)
    assert max_rel(c, ref) <= TOL


@pytest.mark.parametrize("qtype,N", [(F.GGML_TYPE_Q4_K, 512), (F.GGML_TYPE_Q8_0, 512),
                                     (F.GGML_TYPE_Q6_K, 2048)])
@pytest.mark.parametrize("M,K", [(256, 512), (1, 256), (100, 320), (300, 1024), (512, 64)])
def test_gemm_vs_oracle(cuda, oracle, qtype, N, M, K):
    c, ref = _case(cuda, oracle, qtype, M, K, N, M * 7 + K + qtype)
    assert max_rel(c, ref) <= TOL


def test_gemm_bf16_output(cuda, oracle):
    c, ref = _case(cuda, oracle, F.GGML_TYPE_Q4_K, 256, 512, 512, 3, out_dtype=torch.bfloat16)
    assert max_rel(c, ref) <= TOL


def test_gemm_ragged_k_tail(cuda, oracle):
    """K not a multiple of the 64-deep K step: the tail rows come in as zeros."""
    c, ref = _case(cuda, oracle, F.GGML_TYPE_Q8_0, 128, 200, 256, 5)
    assert max_rel(c, ref) <= TOL


# BASELINE config 3 (Q6_K prefill) and config 4/5 shapes at a reduced M
FULL = [(F.GGML_TYPE_Q6_K, 512, 4096, 14336), (F.GGML_TYPE_Q6_K, 512, 14336, 4096),
        (F.GGML_TYPE_Q4_K, 512, 4096, 14336), (F.GGML_TYPE_Q8_0, 256, 8192, 28672)]


@pytest.mark.parametrize("qtype,M,K,N", FULL)
def test_gemm_full_size_vs_fp32_matmul(cuda, qtype, M, K, N):
    w = synthetic_weights(K, N, qtype, seed=0, device=cuda)
    g = torch.Generator(device=cuda).manual_seed(2)
    a = torch.randn(M, K, generator=g, device=cuda).to(torch.bfloat16)
    c = vb.gemm_dequant(a, w, None, M, K, N, qtype)
    deq = vb.dequantize(w, K, N, qtype)  # bit-exact with the reference
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ref = a.float() @ deq
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    err = ((c - ref).abs().max() / ref.abs().max()).item()
    assert err <= TOL
    assert vb.device_status() == 0
    # deterministic: the same inputs give the same bits
    c2 = vb.gemm_dequant(a, w, None, M, K, N, qtype)
    assert torch.equal(c, c2)


def test_gemm_rejects_bad_shapes(cuda):
    a = torch.zeros(4, 64, dtype=torch.bfloat16, device=cuda)
    w = torch.zeros(64 * 144, dtype=torch.uint8, device=cuda)
    with pytest.raises(vb.VbqError, match="multiple of 256"):
        vb.gemm_dequant(a, w, None, 4, 64, 300, "Q4_K")
    w6 = torch.zeros(64 * 210 * 4, dtype=torch.uint8, device=cuda)
    with pytest.raises(vb.VbqError, match="16 bytes"):
        vb.gemm_dequant(a, w6, None, 4, 64, 1024, "Q6_K")


# Several 512-row pair tiles and several waves of the 74 CTA pairs: config 3's M = 2048
# and M = 8192 (the benched sizes; M = 8192 is where the raw-weight ring race once
# showed), Q4_K at M = 8192, and ragged M that ends inside a pair tile and inside a
# CTA's 128-row quarter.
MULTI = [(F.GGML_TYPE_Q6_K, 2048, 4096, 14336), (F.GGML_TYPE_Q6_K, 2048, 14336, 4096),
         (F.GGML_TYPE_Q6_K, 2048, 4096, 6144), (F.GGML_TYPE_Q6_K, 8192, 4096, 14336),
         (F.GGML_TYPE_Q6_K, 8192, 14336, 4096), (F.GGML_TYPE_Q4_K, 8192, 4096, 14336),
         (F.GGML_TYPE_Q4_K, 1573, 4096, 14336), (F.GGML_TYPE_Q4_K, 2000, 14336, 4096),
         (F.GGML_TYPE_Q8_0, 2048 + 37, 8192, 10240)]


@pytest.mark.parametrize("qtype,M,K,N", MULTI)
def test_gemm_multi_tile_vs_fp32_matmul(cuda, qtype, M, K, N):
    """Two bars: the north star's 2e-2 against an fp32 product of the bit-exact
    dequantization, and 1e-4 against the same product over the weights rounded to bf16
    (the kernel's operands), which only accumulation order separates, so a wrong or stale
    tile anywhere in the grid shows.  Three calls give the same bits and a clean status."""
    w = synthetic_weights(K, N, qtype, seed=7, device=cuda)
    g = torch.Generator(device=cuda).manual_seed(8)
    a = torch.randn(M, K, generator=g, device=cuda).to(torch.bfloat16)
    c = vb.gemm_dequant(a, w, None, M, K, N, qtype)
    deq = vb.dequantize(w, K, N, qtype)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        af = a.float()
        ref = af @ deq
        den = ref.abs().max()
        assert ((c - ref).abs().max() / den).item() <= TOL
        del ref
        ref_b = af @ deq.to(torch.bfloat16).float()
        assert ((c - ref_b).abs().max() / den).item() <= 1e-4
        del ref_b
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    assert vb.device_status() == 0
    for _ in range(2):
        c2 = vb.gemm_dequant(a, w, None, M, K, N, qtype)
        assert torch.equal(c, c2)
    assert vb.device_status() == 0


def test_gemm_multi_tile_bf16_out_matches_fp32_out(cuda):
    """bf16 output at M = 8192 is the fp32 output rounded to nearest-even, tile by tile."""
    qtype, M, K, N = F.GGML_TYPE_Q6_K, 8192, 4096, 6144
    w = synthetic_weights(K, N, qtype, seed=9, device=cuda)
    g = torch.Generator(device=cuda).manual_seed(10)
    a = torch.randn(M, K, generator=g, device=cuda).to(torch.bfloat16)
    c32 = vb.gemm_dequant(a, w, None, M, K, N, qtype)
    c16 = vb.gemm_dequant(a, w, None, M, K, N, qtype, out_dtype=torch.bfloat16)
    assert torch.equal(c16, c32.to(torch.bfloat16))
    assert vb.device_status() == 0


# ---- gate | up GEMM fused with SwiGLU (vbq_gemm_swiglu) ----

SWIGLU_CASES = [(F.GGML_TYPE_Q4_K, 2048, 4096, 14336), (F.GGML_TYPE_Q6_K, 1000, 4096, 14336),
                (F.GGML_TYPE_Q8_0, 2048, 8192, 3584), (F.GGML_TYPE_Q4_K, 300, 512, 512),
                (F.GGML_TYPE_Q8_0, 1536 + 37, 1024, 768)]


@pytest.mark.parametrize("qtype,M,K,I", SWIGLU_CASES)
def test_gemm_swiglu_matches_unfused(cuda, qtype, M, K, I):
    """The fused call gives the bits of gate and up GEMMs with bf16 output followed by
    vbq_swiglu (cpp/src/fast_model.cpp:906-953), for separate gate and up matrices and for
    one gate | up matrix packed side by side; repeats are bit-identical."""
    wg = synthetic_weights(K, I, qtype, seed=11, device=cuda)
    wu = synthetic_weights(K, I, qtype, seed=12, device=cuda)
    g = torch.Generator(device=cuda).manual_seed(M + K)
    a = torch.randn(M, K, generator=g, device=cuda).to(torch.bfloat16)
    gate = vb.gemm_dequant(a, wg, None, M, K, I, qtype, out_dtype=torch.bfloat16)
    up = vb.gemm_dequant(a, wu, None, M, K, I, qtype, out_dtype=torch.bfloat16)
    ref = swiglu(gate, up)
    h = vb.gemm_swiglu(a, wg, wu, None, M, K, I, qtype)
    torch.cuda.synchronize()
    assert vb.device_status() == 0
    assert torch.equal(h, ref)
    rb = F.row_bytes(qtype, I)
    packed = torch.cat([wg.view(K, rb), wu.view(K, rb)], dim=1).contiguous()
    h2 = vb.gemm_swiglu(a, packed, packed.view(-1)[rb:], None, M, K, I, qtype, row_bytes=2 * rb)
    assert torch.equal(h2, ref)
    assert torch.equal(vb.gemm_swiglu(a, wg, wu, None, M, K, I, qtype), h)
    # and against fp32 math on the exact dequantized weights (the prefill bar)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        af = a.float()
        gf = af @ vb.dequantize(wg, K, I, qtype)
        uf = af @ vb.dequantize(wu, K, I, qtype)
        hf = torch.nn.functional.silu(gf) * uf
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    assert max_rel(h.float().cpu().numpy(), hf.cpu().numpy()) <= TOL
    assert vb.device_status() == 0
