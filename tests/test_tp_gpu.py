"""Tensor-parallel FFN on the GPU, BASELINE config 5 shapes (70B: hidden 8192,
intermediate 28672, Q8_0).

* One GPU: every rank's shard of TP = 2, 4, 8 runs on cuda:0 and the row-split partial
  sums are added on the device; the result must match TP = 1 and an fp32 torch reference
  over the bit-exact dequantized weights (2e-2 for the bf16 prefill path, 1e-3 for the
  fp32 decode path).
* Two or more GPUs: one process per GPU with NCCL (the all-reduce inside TPFFN); every
  rank must hold the same output, equal to the single-GPU TP = 1 result within the
  tolerance.  Skipped when fewer than two GPUs are visible.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch

import vibeblade_b200 as vb
from vibeblade_b200 import formats as F
from vibeblade_b200 import tp
from vibeblade_b200.quantize import synthetic_weights

pytestmark = pytest.mark.gpu

H, I = 8192, 28672
QT = F.GGML_TYPE_Q8_0


def _weights(dev):
    return (synthetic_weights(H, I, QT, seed=51, device=dev), synthetic_weights(H, I, QT, seed=52, device=dev),
            synthetic_weights(I, H, QT, seed=53, device=dev))


def _rel(a, b):
    return ((a - b).abs().max() / b.abs().max()).item()


@pytest.fixture(scope="module")
def ffn_setup(cuda):
    wg, wu, wd = _weights(cuda)
    g = torch.Generator(device=cuda).manual_seed(2)
    x = torch.randn(256, H, generator=g, device=cuda)
    # fp32 torch reference over the bit-exact dequantization (TF32 off)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        xb = x.to(torch.bfloat16).float()
        G = vb.dequantize(wg, H, I, QT)
        gp = xb @ G
        gd = x[:4] @ G
        del G
        U = vb.dequantize(wu, H, I, QT)
        up = xb @ U
        ud = x[:4] @ U
        del U
        hp = (torch.nn.functional.silu(gp.to(torch.bfloat16).float()) * up.to(torch.bfloat16).float())
        hp = hp.to(torch.bfloat16).float()
        hd = torch.nn.functional.silu(gd) * ud
        D = vb.dequantize(wd, I, H, QT)
        ref_p, ref_d = hp @ D, hd @ D
        del D
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    return wg, wu, wd, x, ref_p, ref_d


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_tp_ffn_prefill_emulated(cuda, ffn_setup, world):
    wg, wu, wd, x, ref_p, _ = ffn_setup
    xb = x.to(torch.bfloat16)
    y = torch.zeros(256, H, device=cuda)
    for r in range(world):  # no process group: each rank's partial sum, added here
        y += tp.TPFFN(wg, wu, wd, H, I, QT, r, world, cuda).prefill(xb, reduce=False)
    torch.cuda.synchronize()
    assert vb.device_status() == 0
    assert _rel(y, ref_p) <= 2e-2


@pytest.mark.parametrize("world", [1, 2, 8])
def test_tp_ffn_decode_emulated(cuda, ffn_setup, world):
    wg, wu, wd, x, _, ref_d = ffn_setup
    y = torch.zeros(4, H, device=cuda)
    for r in range(world):
        y += tp.TPFFN(wg, wu, wd, H, I, QT, r, world, cuda).decode(x[:4].contiguous(), reduce=False)
    torch.cuda.synchronize()
    assert _rel(y, ref_d) <= 1e-3


def test_tp_attention_projections_emulated(cuda):
    """Q / K / V column split by heads (K / V replicated at TP = 8), o row split."""
    KV = 1024  # 8 KV heads x 128
    wq, wk, wv = (synthetic_weights(H, H, QT, seed=61, device=cuda), synthetic_weights(H, KV, QT, seed=62, device=cuda),
                  synthetic_weights(H, KV, QT, seed=63, device=cuda))
    wo = synthetic_weights(H, H, QT, seed=64, device=cuda)
    g = torch.Generator(device=cuda).manual_seed(4)
    x = torch.randn(128, H, generator=g, device=cuda).to(torch.bfloat16)
    full = tp.TPAttentionProj(wq, wk, wv, wo, H, KV, QT, 0, 1, cuda)
    q1, k1, v1 = full.qkv_prefill(x)
    o1 = full.o_prefill(q1)  # any [M, H] bf16 input stands in for the attention output
    for world in (2, 4, 8):
        parts = [tp.TPAttentionProj(wq, wk, wv, wo, H, KV, QT, r, world, cuda) for r in range(world)]
        assert parts[0].kv_replicated == (world == 8)
        q = torch.cat([p.qkv_prefill(x)[0] for p in parts], dim=1)
        assert torch.equal(q, q1)  # column split: identical per-column results
        k = torch.cat([p.qkv_prefill(x)[1] for p in parts], dim=1) if world < 8 else parts[3].qkv_prefill(x)[1]
        assert torch.equal(k, k1)
        hq = H // world
        o = sum(p.o_prefill(q1[:, r * hq:(r + 1) * hq].contiguous(), reduce=False) for r, p in enumerate(parts))
        assert _rel(o, o1) <= 1e-5
    assert vb.device_status() == 0


@pytest.mark.parametrize("world", [1, 8])
def test_tp_ffn_prefill_emulated_m2048(cuda, world):
    """Config 5's prefill size: 2048 rows = four 512-row pair tiles per GEMM, and at TP = 8
    the gate|up GEMM's 1.5 waves.  Same bar and reference as above, plus bit-identical
    repeats."""
    wg, wu, wd = _weights(cuda)
    g = torch.Generator(device=cuda).manual_seed(12)
    M = 2048
    xb = torch.randn(M, H, generator=g, device=cuda).to(torch.bfloat16)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        xf = xb.float()
        gp = (xf @ vb.dequantize(wg, H, I, QT)).to(torch.bfloat16).float()
        up = (xf @ vb.dequantize(wu, H, I, QT)).to(torch.bfloat16).float()
        hp = (torch.nn.functional.silu(gp) * up).to(torch.bfloat16).float()
        del gp, up
        ref = hp @ vb.dequantize(wd, I, H, QT)
        del hp
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    ranks = [tp.TPFFN(wg, wu, wd, H, I, QT, r, world, cuda) for r in range(world)]
    y = torch.zeros(M, H, device=cuda)
    for f in ranks:
        y += f.prefill(xb, reduce=False)
    torch.cuda.synchronize()
    assert vb.device_status() == 0
    assert _rel(y, ref) <= 2e-2
    y2 = torch.zeros(M, H, device=cuda)
    for f in ranks:
        y2 += f.prefill(xb, reduce=False)
    assert torch.equal(y, y2)


def _nccl_rank(rank, world, port, res):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    from datetime import timedelta
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    try:
        wg, wu, wd = _weights(dev)
        g = torch.Generator(device=dev).manual_seed(2)
        # 1024 rows: the FFN runs in two 512-row halves, the first half's all-reduce in
        # flight under the second half's GEMMs
        x = torch.randn(1024, H, generator=g, device=dev).to(torch.bfloat16)
        y = tp.TPFFN(wg, wu, wd, H, I, QT, rank, world, dev).prefill(x)
        ys = [torch.empty_like(y) for _ in range(world)]
        dist.all_gather(ys, y)
        same = all(torch.equal(ys[0], t) for t in ys)
        rel = None
        if rank == 0:  # TP = 1 layer: no collective (reduce_partial follows the layer width)
            y1 = tp.TPFFN(wg, wu, wd, H, I, QT, 0, 1, dev).prefill(x)
            rel = _rel(y, y1)
        torch.cuda.synchronize()
        res[rank] = (same, rel)
        dist.barrier()  # every rank takes the same collective steps before teardown
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_tp_ffn_nccl():
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 8)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    res = mp.get_context("spawn").Manager().dict()
    mp.spawn(_nccl_rank, args=(world, port, res), nprocs=world, join=True)
    assert len(res) == world and all(v[0] for v in res.values())
    assert res[0][1] <= 2e-2
