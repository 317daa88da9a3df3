"""The one-shot all-reduce over peer memory (vbq_peer_allreduce, vibeblade_b200/peer.py).

* One GPU, no waiting: the kernel's sum and publish paths with world = 3 emulated in local
  buffers whose flags are already set, so nothing waits on another launch.  The sum must
  be ((d0 + d1) + d2), the same bits as the rank-order sum on the host side of torch, and
  the kernel must have published the epoch into slot `rank` of every flag array.
* One GPU, the bounded wait: a peer flag that nothing sets; the wait gives up after a short
  budget, the status reports VBQ_ERR_TIMEOUT and the context stays usable.
* Two or more GPUs: one process per GPU (NCCL with NVLS off for the set-up collectives);
  several calls against NCCL's all-reduce of the same partials, every rank holding the
  same bits, and the tensor-parallel FFN decode with the peer all-reduce against the
  collective.  Skipped when fewer than two GPUs are visible.
"""
from __future__ import annotations

import ctypes as C
import os
import socket

import pytest
import torch

import vibeblade_b200 as vb
from vibeblade_b200 import _lib

pytestmark = pytest.mark.gpu


def _ptrs(ts):
    return (C.c_void_p * len(ts))(*[t.data_ptr() for t in ts])


def test_peer_allreduce_rank_order_single_gpu(cuda):
    lib = _lib.load()
    world, rank, epoch, n = 3, 0, 5, 4096 + 3
    g = torch.Generator(device=cuda).manual_seed(1)
    data = [torch.randn(n, generator=g, device=cuda) for _ in range(world)]
    flags = [torch.zeros(8, dtype=torch.int32, device=cuda) for _ in range(world)]
    flags[rank][:world] = epoch  # every peer has published this epoch already
    out = torch.empty(n, device=cuda)
    st = torch.cuda.current_stream(cuda).cuda_stream
    _lib.check(lib.vbq_peer_allreduce(_ptrs(data), _ptrs(flags), world, rank, epoch, n,
                                      C.c_void_p(out.data_ptr()), 0, C.c_void_p(st)), lib)
    torch.cuda.synchronize()
    assert vb.device_status() == 0
    assert torch.equal(out, (data[0] + data[1]) + data[2])
    for p in range(world):  # published into slot `rank` of every rank's flags
        assert int(flags[p][rank].item()) == epoch


def test_peer_allreduce_timeout_reports_status(cuda):
    lib = _lib.load()
    world, rank, epoch, n = 2, 0, 1, 1024
    data = [torch.ones(n, device=cuda) for _ in range(world)]
    flags = [torch.zeros(8, dtype=torch.int32, device=cuda) for _ in range(world)]
    out = torch.zeros(n, device=cuda)
    st = torch.cuda.current_stream(cuda).cuda_stream
    vb.device_status()  # clear
    # rank 1 never publishes: the wait gives up after ~1e6 SM cycles (< 1 ms)
    _lib.check(lib.vbq_peer_allreduce(_ptrs(data), _ptrs(flags), world, rank, epoch, n,
                                      C.c_void_p(out.data_ptr()), 1000000, C.c_void_p(st)), lib)
    torch.cuda.synchronize()
    assert vb.device_status() & 1  # the timeout bit, reported and cleared
    assert torch.count_nonzero(out) == 0  # nothing written after the give-up
    # the context still works
    x = torch.arange(8, device=cuda, dtype=torch.float32)
    assert float((x * 2).sum().item()) == 56.0
    assert vb.device_status() == 0


def _peer_rank(rank, world, port, res):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    from datetime import timedelta
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    par = None
    try:
        from vibeblade_b200.peer import PeerAllReduce
        B, N = 4, 8192
        par = PeerAllReduce(None, B * N, dev)
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        worst, same = 0.0, True
        for call in range(6):
            b = 1 + call % B
            y = par.slot(b, N)
            y.copy_(torch.randn(b, N, generator=g, device=dev))
            ref = y.clone()
            dist.all_reduce(ref)
            out = par.allreduce(y)
            worst = max(worst, float(((out - ref).abs().max() / ref.abs().max()).item()))
            outs = [torch.empty_like(out) for _ in range(world)]
            dist.all_gather(outs, out)
            same = same and all(torch.equal(outs[0], o) for o in outs)
        # tensor-parallel FFN decode (70B shapes, Q8_0): peer all-reduce against the collective
        from vibeblade_b200 import formats as F
        from vibeblade_b200 import tp
        from vibeblade_b200.quantize import synthetic_weights
        H, I, QT = 8192, 28672, F.GGML_TYPE_Q8_0
        wg = synthetic_weights(H, I, QT, seed=1, device=dev)
        wu = synthetic_weights(H, I, QT, seed=2, device=dev)
        wd = synthetic_weights(I, H, QT, seed=3, device=dev)
        f_nccl = tp.TPFFN(wg, wu, wd, H, I, QT, rank, world, dev)
        f_peer = tp.TPFFN(wg, wu, wd, H, I, QT, rank, world, dev)
        f_peer.attach_peer(4, dev)
        x = torch.randn(2, H, generator=torch.Generator(device=dev).manual_seed(7), device=dev)
        y_n = f_nccl.decode(x)
        y_p = f_peer.decode(x)
        y_p2 = f_peer.decode(x)
        ffn_rel = float(((y_p - y_n).abs().max() / y_n.abs().max()).item())
        ffn_rep = bool(torch.equal(y_p, y_p2))
        torch.cuda.synchronize()
        status = vb.device_status()
        res[rank] = (worst, same, ffn_rel, ffn_rep, status)
        f_peer.peer.close()
        dist.barrier()
    finally:
        if par is not None and par._imported:
            par.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_peer_allreduce_multi_gpu():
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 8)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    res = mp.get_context("spawn").Manager().dict()
    mp.spawn(_peer_rank, args=(world, port, res), nprocs=world, join=True)
    assert len(res) == world
    for r, (worst, same, ffn_rel, ffn_rep, status) in res.items():
        assert status == 0, f"rank {r}: device status {status}"
        assert worst <= 1e-6, f"rank {r}: differs from NCCL by {worst}"  # summation order only
        assert same, f"rank {r}: ranks hold different bits"
        assert ffn_rel <= 1e-5, f"rank {r}: FFN decode differs from the collective by {ffn_rel}"
        assert ffn_rep, f"rank {r}: repeated decode not bit-identical"
