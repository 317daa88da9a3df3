"""The FFN's element-wise steps fused into the matmuls (vbq_gemv_ex, vbq_gemm_ex).

The reference runs them as loops of their own around its gemv_dequant calls:
silu(gate) * up (cpp/src/fast_model.cpp:946-953), the Q/K/V biases (:659-668) and the
residual adds after o and down (:813-824, :990-998).  Fused, each must give what the
unfused sequence gives: the same bits where the fused call runs the same kernel (the
additions happen in the same order on the same fp32 sums), and the GEMV bar against the
fp64 product otherwise."""
from __future__ import annotations

import pytest
import torch

import vibeblade_b200 as vb
from vibeblade_b200 import formats as F
from vibeblade_b200 import tp
from vibeblade_b200.quantize import synthetic_weights

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.double() - b.double()).abs().max() / b.double().abs().max()).item()


# (type, K, N, batch): the tensor-core Q4_K kernel (batch 1-4), the wide one (8, 16), the
# Q8_0 kernel, the scalar Q6_K kernel, the generic kernel (router, ragged Q8_0)
EPI = [(F.GGML_TYPE_Q4_K, 4096, 6144, 1), (F.GGML_TYPE_Q4_K, 4096, 6144, 4),
       (F.GGML_TYPE_Q4_K, 4096, 4096, 8), (F.GGML_TYPE_Q4_K, 4096, 4096, 16),
       (F.GGML_TYPE_Q8_0, 8192, 1024, 3), (F.GGML_TYPE_Q6_K, 4096, 4096, 2),
       (F.GGML_TYPE_Q6_K, 14336, 4096, 24), (F.GGML_TYPE_F32, 4096, 8, 5), (F.GGML_TYPE_Q8_0, 2048, 1184, 2)]


def _weights(qtype, K, N, seed, dev):
    if qtype in F.QUANTIZED:
        return synthetic_weights(K, N, qtype, seed=seed, device=dev)
    g = torch.Generator(device=dev).manual_seed(seed)
    return (torch.randn(K, N, generator=g, device=dev) * 0.05).contiguous().view(torch.uint8)


@pytest.mark.parametrize("qtype,K,N,batch", EPI)
def test_gemv_bias_and_residual_epilogue(cuda, qtype, K, N, batch):
    w = _weights(qtype, K, N, 11, cuda)
    g = torch.Generator(device=cuda).manual_seed(12)
    x = torch.randn(batch, K, generator=g, device=cuda)
    bias = torch.randn(N, generator=g, device=cuda)
    res = torch.randn(batch, N, generator=g, device=cuda)
    y = vb.gemv_dequant(x, w, None, K, N, qtype)
    assert torch.equal(vb.gemv_fused(x, w, None, K, N, qtype, bias=bias), y + bias)
    assert torch.equal(vb.gemv_fused(x, w, None, K, N, qtype, residual=res), y + res)
    assert torch.equal(vb.gemv_fused(x, w, None, K, N, qtype, bias=bias, residual=res), (y + bias) + res)
    # in place: the residual stream updated by the projection (output = input + o_proj)
    h = res.clone()
    vb.gemv_fused(x, w, h, K, N, qtype, residual=h)
    assert torch.equal(h, y + res)
    assert vb.device_status() == 0


@pytest.mark.parametrize("qtype,K,N,batch", [(F.GGML_TYPE_Q4_K, 14336, 4096, 1), (F.GGML_TYPE_Q4_K, 14336, 4096, 4),
                                             (F.GGML_TYPE_Q4_K, 14336, 4096, 12), (F.GGML_TYPE_Q8_0, 28672, 8192, 1),
                                             (F.GGML_TYPE_Q8_0, 28672, 8192, 4), (F.GGML_TYPE_Q6_K, 14336, 4096, 3),
                                             (F.GGML_TYPE_Q8_0, 1024, 1184, 6)])
def test_gemv_swiglu_input(cuda, qtype, K, N, batch):
    """The down projection reading silu(gate) * up straight from the gate | up matmul's
    [B, 2K] output: equal to vbq_swiglu_rows followed by the plain GEMV (the same bits on
    the same kernel; batch > 4 Q4_K runs grouped by 4 instead of on the wide kernel, so
    there the GEMV bar), and within 1e-3 of the fp64 product."""
    w = _weights(qtype, K, N, 21, cuda)
    g = torch.Generator(device=cuda).manual_seed(22)
    gu = torch.randn(batch, 2 * K, generator=g, device=cuda) * 3
    res = torch.randn(batch, N, generator=g, device=cuda)
    h = tp.swiglu_rows(gu, K)
    y_ref = vb.gemv_dequant(h, w, None, K, N, qtype)
    y = vb.gemv_fused(gu, w, None, K, N, qtype, swiglu_input=True)
    if qtype == F.GGML_TYPE_Q4_K and batch > 4:
        assert _rel(y, y_ref) <= 1e-5
    else:
        assert torch.equal(y, y_ref)
    ref64 = h.double() @ vb.dequantize(w, K, N, qtype).double()
    assert _rel(y, ref64) <= 1e-3
    y2 = vb.gemv_fused(gu, w, None, K, N, qtype, swiglu_input=True, residual=res)
    assert torch.equal(y2, y + res)
    assert vb.device_status() == 0


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("qtype,M,K,N", [(F.GGML_TYPE_Q4_K, 1000, 4096, 6144), (F.GGML_TYPE_Q8_0, 2048, 8192, 8192),
                                         (F.GGML_TYPE_Q6_K, 300, 4096, 4096)])
def test_gemm_bias_and_residual_epilogue(cuda, qtype, M, K, N, out_dtype):
    """Prefill: bias and residual added to the fp32 accumulator before the one rounding to
    the output type, equal to the fp32 GEMM followed by the adds and that rounding."""
    w = synthetic_weights(K, N, qtype, seed=31, device=cuda)
    g = torch.Generator(device=cuda).manual_seed(32)
    a = torch.randn(M, K, generator=g, device=cuda).to(torch.bfloat16)
    bias = torch.randn(N, generator=g, device=cuda)
    res = torch.randn(M, N, generator=g, device=cuda).to(out_dtype)
    c32 = vb.gemm_dequant(a, w, None, M, K, N, qtype)
    want = ((c32 + bias) + res.float()).to(out_dtype)
    got = vb.gemm_dequant(a, w, None, M, K, N, qtype, out_dtype=out_dtype, bias=bias, residual=res)
    assert torch.equal(got, want)
    inplace = res.clone()
    vb.gemm_dequant(a, w, inplace, M, K, N, qtype, out_dtype=out_dtype, residual=inplace)
    assert torch.equal(inplace, (c32 + res.float()).to(out_dtype))
    assert vb.device_status() == 0
