"""One-shot all-reduce of a row-split layer's fp32 partial over NVLink peer memory.

Tensor parallelism at decode splits o and down by rows (tp.py), so each rank's GEMV leaves
a partial output of B x N floats to be summed over the ranks; the reference runs those
layers whole on one device (cpp/src/fast_model.cpp:813-824, :990-998).  Instead of a
general collective, each rank's GEMV writes its partial into a buffer every peer maps
through CUDA IPC, and one small kernel per rank (vbq_peer_allreduce) publishes the call's
epoch to every peer, waits for theirs (bounded) and sums the partials in rank order, so
all ranks get the same bits.

Set-up is collective (every rank of the group constructs the object with the same
max_floats, then calls allreduce() the same number of times in the same order).  The
buffer is double-buffered by the epoch's parity: write call e's partial into
``slot(B, N)`` (taken before the call), then ``allreduce(y_slot, out)``.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib

FLAG_INTS = 8  # one int32 per possible rank


class PeerAllReduce:
    def __init__(self, group, max_floats: int, device: torch.device):
        import torch.distributed as dist
        self.lib = _lib.load()
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if not 1 <= self.world <= FLAG_INTS:
            raise ValueError(f"PeerAllReduce supports 1..{FLAG_INTS} ranks, got {self.world}")
        self.device = torch.device(device)
        self.cap = (max_floats + 3) // 4 * 4
        # two data slots, then the flag array (int32 view of the last FLAG_INTS floats)
        self.buf = torch.zeros(2 * self.cap + FLAG_INTS, dtype=torch.float32, device=self.device)
        torch.cuda.synchronize(self.device)
        # Every rank takes the same collective steps whatever fails, and all ranks raise
        # together: a failure on one rank must not leave the others in a collective.
        handle = (C.c_char * 64)()
        off = C.c_int64()
        info = None
        with torch.cuda.device(self.device):
            if self.lib.vbq_ipc_export(C.c_void_p(self.buf.data_ptr()), handle, C.byref(off)) == _lib.VBQ_OK:
                info = (bytes(handle), int(off.value))
        infos = [None] * self.world
        dist.all_gather_object(infos, info, group=group)
        if any(i is None for i in infos):
            raise RuntimeError("PeerAllReduce: CUDA IPC export failed on rank(s) "
                               f"{[p for p, i in enumerate(infos) if i is None]}")
        self._imported = []  # (ptr, offset) of the peers' buffers mapped here
        bases = []
        ok = True
        with torch.cuda.device(self.device):
            for p in range(self.world):
                if p == self.rank:
                    bases.append(self.buf.data_ptr())
                    continue
                hp = (C.c_char * 64).from_buffer_copy(infos[p][0])
                ptr = C.c_void_p()
                if self.lib.vbq_ipc_import(hp, infos[p][1], C.byref(ptr)) != _lib.VBQ_OK:
                    ok = False
                    break
                self._imported.append((ptr.value, infos[p][1]))
                bases.append(ptr.value)
        flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=self.device)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
        if int(flag.item()) == 0:
            self.close()
            raise RuntimeError("PeerAllReduce: CUDA IPC import failed on some rank")
        self._bases = bases
        self._flags = (C.c_void_p * self.world)(*[b + 2 * self.cap * 4 for b in bases])
        self._data = [(C.c_void_p * self.world)(*[b + s * self.cap * 4 for b in bases]) for s in range(2)]
        self.epoch = 0
        self.group = group
        dist.barrier(group=group)  # every rank has mapped every buffer before the first call

    def slot(self, B: int, N: int) -> torch.Tensor:
        """This rank's buffer for the next call's partial, as an fp32 [B, N] view."""
        if B * N > self.cap:
            raise ValueError(f"partial of {B * N} floats exceeds the buffer's {self.cap}")
        s = (self.epoch + 1) & 1
        return self.buf[s * self.cap: s * self.cap + B * N].view(B, N)

    def allreduce(self, partial: torch.Tensor, out: torch.Tensor | None = None,
                  timeout_cycles: int = 0) -> torch.Tensor:
        """out = sum over ranks of `partial`, which must be this call's slot()."""
        self.epoch += 1
        s = self.epoch & 1
        if partial.data_ptr() != self.buf.data_ptr() + s * self.cap * 4:
            raise ValueError("partial must be the view returned by slot() for this call")
        if out is None:
            out = torch.empty_like(partial)
        n = partial.numel()
        st = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check(self.lib.vbq_peer_allreduce(self._data[s], self._flags, self.world, self.rank,
                                               self.epoch, n, C.c_void_p(out.data_ptr()),
                                               timeout_cycles, C.c_void_p(st)), self.lib)
        return out

    def close(self) -> None:
        """Unmap the peers' buffers (after every call using them has finished)."""
        torch.cuda.synchronize(self.device)
        with torch.cuda.device(self.device):
            for ptr, off in self._imported:
                _lib.check(self.lib.vbq_ipc_close(C.c_void_p(ptr), off), self.lib)
        self._imported = []
