"""Tensor-parallel host logic on CPU: shard byte layout and split rules, and a
world-size-2 gloo run of the Megatron FFN decomposition (column-split gate / up,
row-split down, one all-reduce) with the oracle's dequantization standing in for the
device kernels."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

from conftest import max_rel
from vibeblade_b200 import formats as F
from vibeblade_b200 import tp
from vibeblade_b200.quantize import quantize

TYPES = [F.GGML_TYPE_Q4_K, F.GGML_TYPE_Q6_K, F.GGML_TYPE_Q8_0]


def _w(K, N, qt, seed):
    return quantize(np.random.default_rng(seed).normal(0, 0.02, (K, N)).astype(np.float32), qt)


@pytest.mark.parametrize("qt", TYPES)
@pytest.mark.parametrize("world", [2, 4])
def test_column_shard_is_column_slice(oracle, qt, world):
    K, N = 16, 4096 * world // 2 if qt == F.GGML_TYPE_Q6_K else 512 * world
    w = _w(K, N, qt, 1)
    full = oracle.dequantize(w.numpy(), K, N, qt)
    n = N // world
    for r in range(world):
        s = tp.shard(w, K, N, qt, "column", r, world)
        assert s.shape == (K, F.row_bytes(qt, n))
        np.testing.assert_array_equal(oracle.dequantize(s.numpy(), K, n, qt), full[:, r * n:(r + 1) * n])


@pytest.mark.parametrize("qt", TYPES)
def test_row_shard_is_row_slice(oracle, qt):
    K, N, world = 64, 2048, 4
    w = _w(K, N, qt, 2)
    full = oracle.dequantize(w.numpy(), K, N, qt)
    k = K // world
    for r in range(world):
        s = tp.shard(w, K, N, qt, "row", r, world)
        np.testing.assert_array_equal(oracle.dequantize(s.numpy(), k, N, qt), full[r * k:(r + 1) * k])


@pytest.mark.parametrize("qt,H,I", [(F.GGML_TYPE_Q8_0, 256, 1024), (F.GGML_TYPE_Q4_K, 256, 1024),
                                    (F.GGML_TYPE_Q6_K, 256, 8192)])
def test_packed_gate_up_is_side_by_side_shards(oracle, qt, H, I):
    """The FFN's packed gate | up matrix of a rank: each row is the gate shard's blocks then
    the up shard's, so its dequantization is the two shards' dequantizations side by side."""
    rng = np.random.default_rng(qt)
    wg = quantize(rng.normal(0, 0.02, (H, I)).astype(np.float32), qt)
    wu = quantize(rng.normal(0, 0.02, (H, I)).astype(np.float32), qt)
    for world in (1, 2, 4):
        for r in range(world):
            gs, us = (tp.shard(w, H, I, qt, "column", r, world) for w in (wg, wu))
            lin = tp.TPLinear.packed_columns([gs, us], H, qt, torch.device("cpu"))
            n = I // world
            assert (lin.k_loc, lin.n_loc) == (H, 2 * n)
            full = oracle.dequantize(lin.w.numpy(), H, 2 * n, qt)
            np.testing.assert_array_equal(full[:, :n], oracle.dequantize(gs.numpy(), H, n, qt))
            np.testing.assert_array_equal(full[:, n:], oracle.dequantize(us.numpy(), H, n, qt))


def test_split_rules():
    # 70B shapes (hidden 8192, intermediate 28672, Q8_0) split at 1, 2, 4, 8
    for world in (1, 2, 4, 8):
        tp.check_split("column", 8192, 28672, F.GGML_TYPE_Q8_0, world)
        tp.check_split("row", 28672, 8192, F.GGML_TYPE_Q8_0, world)
        tp.check_split("column", 8192, 8192, F.GGML_TYPE_Q8_0, world)
    tp.check_split("column", 8192, 1024, F.GGML_TYPE_Q8_0, 4)
    with pytest.raises(ValueError):  # 8 KV heads x 128 over 8 ranks: 128 columns each
        tp.check_split("column", 8192, 1024, F.GGML_TYPE_Q8_0, 8)
    with pytest.raises(ValueError):
        tp.check_split("row", 100, 256, F.GGML_TYPE_Q4_K, 8)
    with pytest.raises(ValueError):  # Q6_K shard rows must stay 16-byte multiples
        tp.check_split("column", 64, 2048, F.GGML_TYPE_Q6_K, 2)
    # the types only the generic / staged GEMV read take 2-byte-aligned shard rows: a Q3_K
    # shard of 256 columns is 110 bytes a row, a Q8_K one 292
    tp.check_split("column", 64, 2048, F.GGML_TYPE_Q3_K, 8)
    tp.check_split("column", 64, 512, F.GGML_TYPE_Q8_K, 2)
    with pytest.raises(ValueError):  # whole 256-column tiles still
        tp.check_split("column", 64, 512, F.GGML_TYPE_Q4_0, 4)


def test_column_shards_of_the_other_block_types(oracle):
    """Column shards of the dispatcher's other block types are the same bytes as the
    columns of the whole matrix (block-aligned byte ranges of every row)."""
    from block_fill import TYPES, random_blocks
    rng = np.random.default_rng(5)
    K, N, world = 6, 1024, 2
    for t in TYPES:
        w = torch.from_numpy(random_blocks(t, K, N, rng))
        full = oracle.dequantize(w.numpy(), K, N, t)
        parts = [oracle.dequantize(tp.shard(w, K, N, t, "column", r, world).numpy(), K, N // world, t)
                 for r in range(world)]
        np.testing.assert_array_equal(np.concatenate(parts, axis=1).view(np.uint32), full.view(np.uint32))


def _silu(x):
    return x / (1.0 + np.exp(-x))


def _ffn_rank(rank, world, port, H, I, qt, res):
    import torch.distributed as dist
    from oracle import load_oracle
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        orc = load_oracle()
        wg, wu, wd = _w(H, I, qt, 10), _w(H, I, qt, 11), _w(I, H, qt, 12)
        x = np.random.default_rng(5).normal(0, 1, (3, H))
        il = I // world
        g = x @ orc.dequantize(tp.shard(wg, H, I, qt, "column", rank, world).numpy(), H, il, qt)
        u = x @ orc.dequantize(tp.shard(wu, H, I, qt, "column", rank, world).numpy(), H, il, qt)
        part = (_silu(g) * u) @ orc.dequantize(tp.shard(wd, I, H, qt, "row", rank, world).numpy(), il, H, qt)
        y = torch.from_numpy(part)
        dist.all_reduce(y)
        full = (_silu(x @ orc.dequantize(wg.numpy(), H, I, qt)) * (x @ orc.dequantize(wu.numpy(), H, I, qt))) \
            @ orc.dequantize(wd.numpy(), I, H, qt)
        res[rank] = max_rel(y.numpy(), full)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("qt", [F.GGML_TYPE_Q8_0, F.GGML_TYPE_Q4_K])
def test_tp_ffn_gloo_world2(qt):
    import torch.multiprocessing as mp
    H, I, world = 256, 1024, 2
    res = mp.get_context("spawn").Manager().dict()
    mp.spawn(_ffn_rank, args=(world, _free_port(), H, I, qt, res), nprocs=world, join=True)
    assert len(res) == world
    assert max(res.values()) <= 1e-9  # fp64 sums: only the split of the sum differs


def _reduce_rank(rank, world, port, res):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    try:
        y = torch.full((4,), float(rank + 1))
        # a TP = 1 layer on one rank only: no collective may start
        if rank == 0:
            assert torch.equal(tp.reduce_partial(y.clone(), 1), y)
        # a layer split over a width that is not the group's: refused on every rank
        try:
            tp.reduce_partial(y.clone(), world + 1)
            bad = False
        except RuntimeError:
            bad = True
        s = tp.reduce_partial(y.clone(), world)  # the real split: summed over the ranks
        res[rank] = (bad, s.tolist())
    finally:
        dist.destroy_process_group()


def test_reduce_partial_collective_decision():
    """The all-reduce follows the layer's TP width, not the process group's size: a TP = 1
    call made on one rank of a 2-rank job returns at once (a collective there would hang
    the other rank; the 20 s group timeout turns such a regression into a failure)."""
    import torch.multiprocessing as mp
    res = mp.get_context("spawn").Manager().dict()
    mp.spawn(_reduce_rank, args=(2, _free_port(), res), nprocs=2, join=True)
    assert res[0] == (True, [3.0] * 4) and res[1] == (True, [3.0] * 4)


class _CpuRowLinear:
    """Stand-in for a row-split TPLinear on the CPU: rank r's rows of a dense weight."""

    def __init__(self, w_full: torch.Tensor, rank: int, world: int):
        K = w_full.shape[0]
        self.world, self.n_loc = world, w_full.shape[1]
        self.w = w_full[rank * K // world:(rank + 1) * K // world]

    def prefill(self, a, out_dtype=torch.float32, out=None):
        r = a.float() @ self.w
        if out is None:
            return r
        out.copy_(r)
        return out


def _row_split_rank(rank, world, port, res):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    try:
        g = torch.Generator().manual_seed(5)
        out = {}
        for M in (300, 600, 2048):  # no split, split at 512, split at 1024
            a = torch.randn(M, 64, generator=g)
            w = torch.randn(64, 48, generator=g)
            lin = _CpuRowLinear(w, rank, world)
            k = 64 // world
            a_loc = a[:, rank * k:(rank + 1) * k].contiguous()
            ref = a @ w
            y32 = tp.row_split_prefill_reduced(lin, a_loc, reduce_dtype=torch.float32)
            y16 = tp.row_split_prefill_reduced(lin, a_loc)  # the default: bf16 partial sums
            out[M] = (float((y32 - ref).abs().max()),
                      float((y16 - ref).abs().max() / ref.abs().max()), y16.dtype == torch.float32)
        res[rank] = out
    finally:
        dist.destroy_process_group()


def test_row_split_prefill_reduced_gloo():
    """The row-split prefill with its first half's all-reduce in flight while the second
    half computes (split at whole 512-row pair tiles): the sum over ranks equals the full
    product for M with no split, an uneven split and an even one -- to fp32 rounding with
    fp32 partial sums, within the prefill's 2e-2 bar with the default bf16 ones (returned
    as fp32)."""
    import torch.multiprocessing as mp
    res = mp.get_context("spawn").Manager().dict()
    mp.spawn(_row_split_rank, args=(2, _free_port(), res), nprocs=2, join=True)
    for rank in (0, 1):
        assert all(e32 < 1e-4 and e16 <= 2e-2 and f32 for e32, e16, f32 in res[rank].values()), res[rank]
