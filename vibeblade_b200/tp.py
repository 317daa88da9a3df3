"""Tensor-parallel sharding of quantized weights and the TP FFN / attention projections.

The reference runs on one host (its engine has no multi-GPU path); this module splits the
same matmuls Megatron-style over the GPUs of one node, one process per GPU:

* column split (Q, K, V, gate, up; ``kind="column"``): rank r owns output columns
  [r N / W, (r + 1) N / W).  In the reference block layout (K x N, blocks along N) that
  is the same byte range of every row, so the shard is a strided, block-aligned slice
  packed into its own K x (N / W) matrix.  Outputs are disjoint: no communication.
* row split (o, down; ``kind="row"``): rank r owns input rows [r K / W, (r + 1) K / W):
  a contiguous byte range.  Each rank produces a partial [M, N] sum; one all-reduce (sum)
  over the process group combines them, two per layer (after o and after down).

``TPFFN`` is the SwiGLU FFN of one layer (gate / up column split, down row split);
``TPAttentionProj`` the Q, K/V (column) and o (row) projections around the attention core,
which is outside the quantized matmul path.  Prefill uses the tcgen05 GEMM (bf16
activations), decode the fused GEMV (fp32).  The collective is torch.distributed's
all_reduce on the process group (NCCL between GPUs).

Gate and up (independent column splits over the same x) are one matmul over their packed
shards: one launch instead of two, and at TP >= 4, where each alone fills only part of the
GPU's CTA-pair slots, together they fill 1.5 waves instead of two.  A row-split layer's
GEMM runs in two row halves and the first half's all-reduce (on NCCL's stream) overlaps
the second half's GEMM.
"""
from __future__ import annotations

import torch

from . import _lib
from . import formats as F
from .dequant import _require_cuda, _stream_ptr, _weights_u8, gemv_dequant
from .gemm import gemm_dequant, gemm_swiglu

# GEMM tiles are 256 columns wide; a column shard must keep whole tiles
SHARD_COLUMN_ALIGN = 256


def check_split(kind: str, K: int, N: int, qtype, world: int) -> None:
    t = F.parse_type(qtype)
    if kind == "column":
        if N % world or (N // world) % SHARD_COLUMN_ALIGN or (N // world) % F.BLOCK_VALUES[t]:
            raise ValueError(f"column split: N={N} over {world} ranks must leave multiples of "
                             f"{SHARD_COLUMN_ALIGN} columns per rank")
        # the tiled kernels and the GEMM read rows by TMA (16-byte strides); the generic
        # GEMV, which takes every other block type, reads 2-byte-aligned rows
        if t in F.QUANTIZED and F.row_bytes(t, N // world) % 16:
            raise ValueError("column split: shard rows must be a multiple of 16 bytes "
                             "(Q6_K: N / world % 2048 == 0)")
    elif kind == "row":
        if K % world or (K // world) % 8:
            raise ValueError(f"row split: K={K} over {world} ranks must leave multiples of 8 rows")
    else:
        raise ValueError(kind)


def shard(w: torch.Tensor, K: int, N: int, qtype, kind: str, rank: int, world: int) -> torch.Tensor:
    """Rank `rank`'s shard of the K x N block matrix `w` (uint8 bytes, any device), packed
    as its own block matrix: K x (N / world) for a column split, (K / world) x N for a row
    split."""
    t = F.parse_type(qtype)
    check_split(kind, K, N, t, world)
    rb = F.row_bytes(t, N)
    m = _weights_u8(w).reshape(-1)[:K * rb].view(K, rb)
    if kind == "column":
        per = F.row_bytes(t, N // world)
        return m[:, rank * per:(rank + 1) * per].contiguous()
    kr = K // world
    return m[rank * kr:(rank + 1) * kr].contiguous()


def swiglu_rows(gu: torch.Tensor, n: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """silu(gate) * up for rows of [gate | up] (gu: fp32 or bf16 CUDA [rows, 2n], the output of
    one matmul over gate and up packed side by side) -> [rows, n]."""
    _require_cuda("swiglu_rows", gu)
    if gu.dim() != 2 or gu.shape[1] != 2 * n or gu.dtype not in (torch.float32, torch.bfloat16) \
            or not gu.is_contiguous():
        raise RuntimeError("swiglu_rows: gu must be a contiguous fp32 or bf16 [rows, 2n] tensor")
    out = torch.empty((gu.shape[0], n), dtype=gu.dtype, device=gu.device) if out is None else out
    lib = _lib.load()
    dt = _lib.DTYPE_F32 if gu.dtype == torch.float32 else _lib.DTYPE_BF16
    _lib.check(lib.vbq_swiglu_rows(gu.data_ptr(), out.data_ptr(), gu.shape[0], n, dt,
                                   _stream_ptr(gu)), lib)
    return out


def swiglu(g: torch.Tensor, u: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """silu(g) * u (fp32 or bf16 CUDA tensors, same shape), g and u sanitised first."""
    _require_cuda("swiglu", g, u)
    if g.shape != u.shape or g.dtype != u.dtype or g.dtype not in (torch.float32, torch.bfloat16):
        raise RuntimeError("swiglu: g and u must be fp32 or bf16 tensors of one shape")
    out = torch.empty_like(g) if out is None else out
    lib = _lib.load()
    dt = _lib.DTYPE_F32 if g.dtype == torch.float32 else _lib.DTYPE_BF16
    _lib.check(lib.vbq_swiglu(g.data_ptr(), u.data_ptr(), out.data_ptr(), g.numel(), dt,
                              _stream_ptr(g)), lib)
    return out


class TPLinear:
    """One quantized matmul split over the group: y = x @ deq(W), W K x N."""

    def __init__(self, w_full: torch.Tensor, K: int, N: int, qtype, kind: str, rank: int,
                 world: int, device: torch.device):
        self.t = F.parse_type(qtype)
        self.kind, self.K, self.N, self.rank, self.world = kind, K, N, rank, world
        self.w = shard(w_full, K, N, self.t, kind, rank, world).to(device)
        self.k_loc = K // world if kind == "row" else K
        self.n_loc = N // world if kind == "column" else N

    def prefill(self, a: torch.Tensor, out_dtype=torch.float32,
                out: torch.Tensor | None = None) -> torch.Tensor:
        """a: bf16 [M, k_loc] -> [M, n_loc] (row split: a partial sum).  The tensor-core
        GEMM takes Q4_K / Q6_K / Q8_0; the other types run as one generic GEMV over all M
        rows (fp32 sums, as the reference's per-token loop computes them)."""
        if self.t not in F.QUANTIZED:
            y = gemv_dequant(a.float().contiguous(), self.w, None, self.k_loc, self.n_loc, self.t)
            y = y.view(a.shape[0], self.n_loc).to(out_dtype)
            if out is None:
                return y
            out.copy_(y)
            return out
        return gemm_dequant(a, self.w, out, a.shape[0], self.k_loc, self.n_loc, self.t, out_dtype)

    def decode(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """x: fp32 [B, k_loc] (B <= 32) -> fp32 [B, n_loc] (into `out` when given)."""
        return gemv_dequant(x, self.w, out, self.k_loc, self.n_loc, self.t)

    @classmethod
    def packed_columns(cls, parts, K: int, qtype, device: torch.device) -> "TPLinear":
        """One matmul over several column-split layers of the same input: the shards
        ``parts`` (uint8 K x row-bytes block matrices of this rank) packed side by side,
        each row holding the parts' blocks in order, so one GEMM / GEMV computes all of
        them and its output columns are the parts' outputs in order."""
        t = F.parse_type(qtype)
        self = cls.__new__(cls)
        self.t, self.kind, self.K, self.rank, self.world = t, "column", K, 0, 1
        self.w = torch.cat([p.reshape(K, -1) for p in parts], dim=1).contiguous().to(device)
        self.N = self.n_loc = self.w.shape[1] // F.BLOCK_BYTES[t] * F.BLOCK_VALUES[t]
        self.k_loc = K
        return self


def reduce_partial(y: torch.Tensor, world: int, group=None, async_op: bool = False):
    """Sum a row-split layer's partial output over its `world` ranks (in place).

    The decision depends only on the layer's own TP width, never on the size of whatever
    process group exists: a TP = 1 layer (for example a single-GPU reference computed on
    one rank of a larger job) must not enter a collective the other ranks do not join.
    A layer split over W > 1 ranks needs a process group of exactly W ranks.  async_op
    returns the collective's work handle (None at W = 1) instead of y."""
    if world == 1:
        return None if async_op else y
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()):
        raise RuntimeError(f"a layer split over {world} ranks needs torch.distributed initialised")
    if dist.get_world_size(group) != world:
        raise RuntimeError(f"layer split over {world} ranks but the process group has "
                           f"{dist.get_world_size(group)}")
    work = dist.all_reduce(y, op=dist.ReduceOp.SUM, group=group, async_op=async_op)
    return work if async_op else y


# rows of a GEMM pair tile: a split at a multiple keeps both halves in whole tiles
_PAIR_TILE_ROWS = 512


def row_split_prefill_reduced(lin: "TPLinear", a: torch.Tensor, group=None,
                              reduce_dtype=torch.bfloat16) -> torch.Tensor:
    """fp32 [M, N] = all-reduce over the ranks of lin.prefill(a) for a row-split layer.

    Over W > 1 ranks the GEMM writes its partial sums in `reduce_dtype` (bf16 by default:
    half the bytes to write and to move over NVLink, within the prefill's bf16 bar) and the
    all-reduce sums them in that type; the result is returned in fp32.  The GEMM runs in
    two row halves (split at whole 512-row pair tiles); the first half's all-reduce is
    issued as soon as its GEMM is enqueued and runs on NCCL's stream while the second half
    computes.  Every rank takes the same collective steps for the same M."""
    M, W = a.shape[0], lin.world
    dt = torch.float32 if W == 1 else reduce_dtype
    y = torch.empty((M, lin.n_loc), dtype=dt, device=a.device)
    split = ((M // 2 + _PAIR_TILE_ROWS - 1) // _PAIR_TILE_ROWS) * _PAIR_TILE_ROWS
    if W == 1 or split >= M:
        lin.prefill(a, dt, out=y)
        reduce_partial(y, W, group)
        return y if dt == torch.float32 else y.float()
    lin.prefill(a[:split], dt, out=y[:split])
    work = reduce_partial(y[:split], W, group, async_op=True)
    lin.prefill(a[split:], dt, out=y[split:])
    reduce_partial(y[split:], W, group)
    work.wait()
    return y if dt == torch.float32 else y.float()


class TPFFN:
    """SwiGLU FFN of one layer: out = down(silu(gate x) * up x), gate / up column split,
    down row split, one all-reduce (cpp/src/fast_model.cpp:906-958).

    The rank's gate and up shards are packed side by side into one K x (2 I / W) matrix
    (no requantisation: each row is the gate shard's blocks, then the up shard's), so one
    GEMM (prefill) or GEMV (decode) launch computes both and SwiGLU reads the two halves
    of each output row (``swiglu_rows``)."""

    def __init__(self, wg, wu, wd, H: int, I: int, qtype, rank: int, world: int, device,
                 group=None):
        t = F.parse_type(qtype)
        check_split("column", H, I, t, world)
        self.i_loc = I // world
        self.gate_up = TPLinear.packed_columns(
            [shard(wg, H, I, t, "column", rank, world), shard(wu, H, I, t, "column", rank, world)],
            H, t, device)
        self.down = TPLinear(wd, I, H, qtype, "row", rank, world, device)
        self.group = group
        self.H = H
        self.peer = None  # PeerAllReduce for decode (attach_peer), else the group's collective
        self.peer_batch = 0

    def attach_peer(self, max_batch: int, device) -> None:
        """Decode's all-reduce over NVLink peer memory (peer.PeerAllReduce) instead of the
        process group's collective, for batches up to max_batch; collective set-up, every
        rank calls it.  The down GEMV then writes its partial straight into the shared
        buffer.  The one-shot reads every peer's whole partial, W times the bytes of a ring,
        so it pays for small partials: measured on 8 B200s (70B FFN decode, us, peer / NCCL)
        batch 1 49.2 / 68.4, batch 16 187.3 / 189.7, batch 32 357.9 / 344.0; 16 is the
        largest batch worth attaching."""
        if self.down.world > 1:
            from .peer import PeerAllReduce
            self.peer = PeerAllReduce(self.group, max_batch * self.H, device)
            self.peer_batch = max_batch

    def prefill(self, x: torch.Tensor, reduce: bool = True) -> torch.Tensor:
        """x: bf16 [M, H] (replicated) -> fp32 [M, H], replicated after the all-reduce
        (reduce=False returns this rank's partial sum and leaves the sum to the caller).

        Over W > 1 ranks the whole FFN runs in two row halves (split at whole 512-row pair
        tiles): the first half's bf16 all-reduce runs on NCCL's stream under the second
        half's gate|up GEMM, SwiGLU and down GEMM, and only the second half's is exposed
        (measured at TP = 8: 0.492 ms per M = 2048 step, against 0.615 ms when only the down
        GEMM is split).  Rows are independent in every step, so the halves give the same
        bits as one pass."""
        W = self.down.world
        M = x.shape[0]
        split = ((M // 2 + _PAIR_TILE_ROWS - 1) // _PAIR_TILE_ROWS) * _PAIR_TILE_ROWS
        if W == 1 or split >= M:
            h = self.gate_up_swiglu(x)
            if not reduce:
                return self.down.prefill(h, torch.float32)
            return row_split_prefill_reduced(self.down, h, self.group)
        dt = torch.bfloat16 if reduce else torch.float32
        y = torch.empty((M, self.down.n_loc), dtype=dt, device=x.device)
        work = None
        for lo, hi in ((0, split), (split, M)):
            h = self.gate_up_swiglu(x[lo:hi])
            self.down.prefill(h, dt, out=y[lo:hi])
            if reduce:
                if work is None:
                    work = reduce_partial(y[lo:hi], W, self.group, async_op=True)
                else:
                    reduce_partial(y[lo:hi], W, self.group)
        if work is not None:
            work.wait()
        return y if dt == torch.float32 else y.float()

    def gate_up_swiglu(self, x: torch.Tensor) -> torch.Tensor:
        """bf16 [M, H] -> bf16 h [M, I / W] = silu(x Wgate) * (x Wup) for this rank's shard: one
        GEMM over the packed gate | up matrix with SwiGLU in its epilogue (vbq_gemm_swiglu),
        where the up part starts on a 16-byte boundary; else the GEMM and a SwiGLU pass."""
        g = self.gate_up
        gate_bytes = F.row_bytes(g.t, self.i_loc)
        if gate_bytes % 16 == 0 and self.i_loc % 256 == 0:
            return gemm_swiglu(x, g.w, g.w.view(-1)[gate_bytes:], None, x.shape[0], g.k_loc, self.i_loc, g.t,
                               row_bytes=2 * gate_bytes)
        return swiglu_rows(g.prefill(x, torch.bfloat16), self.i_loc)

    def decode(self, x: torch.Tensor, reduce: bool = True) -> torch.Tensor:
        """x: fp32 [B, H] -> fp32 [B, H] (reduce as for prefill).  SwiGLU runs as one pass over
        the gate | up output: read inside the down GEMV it would be recomputed by each of the
        GEMV's 256-column tiles (measured on the 70B shard at TP = 1: 48 us plain against 77 us
        fused at batch 1, 304 against 892 at batch 16)."""
        h = swiglu_rows(self.gate_up.decode(x), self.i_loc)
        if reduce and self.peer is not None and x.shape[0] <= self.peer_batch:
            y = self.down.decode(h, out=self.peer.slot(x.shape[0], self.H))
            return self.peer.allreduce(y)
        y = self.down.decode(h)
        return reduce_partial(y, self.down.world, self.group) if reduce else y


class TPAttentionProj:
    """Q, K, V and o projections of one attention layer around the attention core.

    Q, K and V are split by heads (columns), so rank r holds query heads r Hq / W .. and
    the KV heads they attend to.  When a K / V shard would fall below the kernels'
    256-column tiles (8 KV heads of 128 over 8 ranks) each rank computes all KV heads
    instead (replicated).  o is split by rows and followed by the all-reduce."""

    def __init__(self, wq, wk, wv, wo, H: int, kv_cols: int, qtype, rank: int, world: int,
                 device, group=None):
        self.q = TPLinear(wq, H, H, qtype, "column", rank, world, device)
        try:
            check_split("column", H, kv_cols, qtype, world)
            kv_rank, kv_world = rank, world
        except ValueError:
            kv_rank, kv_world = 0, 1
        self.kv_replicated = kv_world == 1 and world > 1
        self.k = TPLinear(wk, H, kv_cols, qtype, "column", kv_rank, kv_world, device)
        self.v = TPLinear(wv, H, kv_cols, qtype, "column", kv_rank, kv_world, device)
        self.o = TPLinear(wo, H, H, qtype, "row", rank, world, device)
        self.group = group

    def qkv_prefill(self, x: torch.Tensor):
        """x: bf16 [M, H] -> bf16 (q [M, H / W], k, v [M, kv_cols / W or kv_cols])."""
        return (self.q.prefill(x, torch.bfloat16), self.k.prefill(x, torch.bfloat16),
                self.v.prefill(x, torch.bfloat16))

    def o_prefill(self, attn: torch.Tensor, reduce: bool = True) -> torch.Tensor:
        """attn: bf16 [M, H / world] (this rank's heads) -> fp32 [M, H] after all-reduce
        (reduce=False: this rank's partial sum)."""
        if not reduce:
            return self.o.prefill(attn, torch.float32)
        return row_split_prefill_reduced(self.o, attn, self.group)
