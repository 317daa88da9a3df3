"""Device SwiGLU (the FFN's silu(gate) * up, cpp/src/fast_model.cpp:946-953, with the
reference MoE path's sanitising, vibeblade/moe.py:36-50, :472-474) against the numpy
restatement in oracle/moe_oracle.py, and the row-wise form over a packed [gate | up]
matmul output against the elementwise one."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.moe_oracle import _sanitize, silu
from vibeblade_b200 import tp

pytestmark = pytest.mark.gpu


def _inputs(rows, n, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(rows, 2 * n, generator=g) * 6
    flat = a.view(-1)
    flat[::97] = float("nan")
    flat[5::211] = float("inf")
    flat[9::307] = -float("inf")
    flat[13::401] = 1e6
    return a


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_swiglu_matches_oracle(cuda, dtype):
    gu = _inputs(8, 1024, 1).to(dtype)
    g, u = gu[:, :1024].contiguous(), gu[:, 1024:].contiguous()
    h = tp.swiglu(g.to(cuda), u.to(cuda)).float().cpu().numpy()
    gf, uf = g.float().numpy(), u.float().numpy()
    ref = silu(_sanitize(gf)) * _sanitize(uf)
    if dtype == torch.bfloat16:  # computed in fp32, rounded once to bf16
        ref = torch.from_numpy(ref.astype(np.float32)).to(torch.bfloat16).float().numpy()
    # the device exp differs from numpy's in the last bit: bounded relative error
    np.testing.assert_allclose(h, ref, rtol=1e-5 if dtype == torch.float32 else 8e-3, atol=1e-30)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("rows,n", [(1, 8), (3, 1024), (16, 3584), (2048, 256)])
def test_swiglu_rows_equals_elementwise(cuda, dtype, rows, n):
    """Rows of [gate | up] (one matmul over the packed gate and up shards) give exactly the
    elementwise result on the two halves."""
    gu = _inputs(rows, n, rows + n).to(dtype).to(cuda)
    h_rows = tp.swiglu_rows(gu, n)
    h_elem = tp.swiglu(gu[:, :n].contiguous(), gu[:, n:].contiguous())
    assert h_rows.shape == (rows, n)
    assert torch.equal(h_rows.view(torch.int16 if dtype == torch.bfloat16 else torch.int32),
                       h_elem.view(torch.int16 if dtype == torch.bfloat16 else torch.int32))


def test_swiglu_rows_rejects_bad_shapes(cuda):
    with pytest.raises(RuntimeError):
        tp.swiglu_rows(torch.zeros(4, 30, device=cuda), 15)   # n not a multiple of 8
    with pytest.raises(RuntimeError):
        tp.swiglu_rows(torch.zeros(4, 32, device=cuda), 8)    # 2n != columns
