"""Engine integration: one transformer block's matmuls on the device, loaded from GGUF.

The reference engine's block, ``VibeBladeFast::forward_layer`` (cpp/src/fast_model.cpp:
578-998; the Python engine's ``forward_token``, vibeblade/transformer.py:232-325), runs

    h = rms_norm(x);  q, k, v = h Wq (+bq), h Wk (+bk), h Wv (+bv)      [:645-668]
    rope, attention over the KV cache                                   [:690-804]
    x = x + attn Wo                                                     [:806-824]
    h = rms_norm(x);  x = x + down(silu(h Wgate) * (h Wup))            [:826-998]
    (MoE layers: router GEMV, top-k, per-expert FFNs)                  [:840-903]

with one ``gemv_dequant`` per token and matrix.  ``DeviceLayer`` replaces every one of
those matmul call sites: the block's quantized weights are uploaded once from the GGUF
file (tensor-parallel shards read straight from the file), Q | K | V and gate | up are
packed into one matrix each (one launch), and the element-wise steps around the matmuls run
inside them -- the biases and the residual adds in the epilogues, SwiGLU as the down
projection's input at decode (vbq_gemv_ex / vbq_gemm_ex).  Decode (up to 32 tokens) runs
the fused GEMV kernels, prefill the tcgen05 GEMM.  Norms, RoPE and attention stay the
engine's: ``forward`` takes the attention as a callable and an optional norm.

Tensor parallelism (Megatron split over the ranks of a process group): Q / K / V and gate /
up by output columns, o and down by input rows; rank 0 adds the residual into its partial
sum and one all-reduce per row-split matmul completes the sum.  K / V are replicated when
their heads do not split into whole 256-column tiles (each rank then keeps the KV heads its
query heads read).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import formats as F
from .dequant import gemv_fused
from .gemm import gemm_dequant, gemm_swiglu
from .gguf import GGUFFile
from .tp import SHARD_COLUMN_ALIGN, swiglu_rows

DECODE_MAX_TOKENS = 32  # the GEMV kernels' batch limit; longer inputs take the GEMM


@dataclass
class LayerConfig:
    """Llama-style block geometry (the GGUF metadata ``<arch>.*`` keys the reference reads in
    VibeBladeFast::extract_config, cpp/src/fast_model.cpp:176-260)."""
    hidden: int
    n_heads: int
    n_kv_heads: int
    ffn: int
    eps: float = 1e-5

    @property
    def head_dim(self) -> int:
        return self.hidden // self.n_heads

    @classmethod
    def from_gguf(cls, f: GGUFFile) -> "LayerConfig":
        arch = f.meta_string("general.architecture") or "llama"
        hidden = f.meta_int(f"{arch}.embedding_length")
        n_heads = f.meta_int(f"{arch}.attention.head_count")
        return cls(hidden=hidden, n_heads=n_heads,
                   n_kv_heads=f.meta_int(f"{arch}.attention.head_count_kv", n_heads),
                   ffn=f.meta_int(f"{arch}.feed_forward_length"),
                   eps=f.meta_float(f"{arch}.attention.layer_norm_rms_epsilon", 1e-5))


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """The reference's RMSNorm (vibeblade/transformer.py:42-61): inputs and weights
    sanitised to the fp16 range, x / max(sqrt(mean(x^2) + eps), eps) * w, result sanitised."""
    def clean(t):
        return torch.nan_to_num(t.float(), nan=0.0, posinf=65504.0, neginf=-65504.0).clamp(-65504.0, 65504.0)
    x32, w32 = clean(x), clean(w)
    rms = torch.sqrt((x32 * x32).mean(dim=-1, keepdim=True) + eps).clamp_min(eps)
    return clean((x32 / rms) * w32)


class DeviceLayer:
    """Block `layer` of a GGUF model on `device`, as rank `rank` of `world`."""

    def __init__(self, f: GGUFFile, layer: int, device, cfg: LayerConfig | None = None,
                 rank: int = 0, world: int = 1, group=None, reduce: bool = True):
        """reduce=False leaves the row-split outputs as this rank's partial sums (all ranks
        emulated on one device add them up)."""
        self.cfg = cfg or LayerConfig.from_gguf(f)
        self.dev = torch.device(device)
        self.rank, self.world, self.group, self.reduce = rank, world, group, reduce
        c = self.cfg
        p = f"blk.{layer}."
        if c.n_heads % world or c.ffn % world:
            raise ValueError(f"heads / ffn do not split over {world} ranks")
        self.q_heads = c.n_heads // world
        # K / V split with Q when their shard is whole tiles, else replicated
        kv_split = c.n_kv_heads % world == 0 and (c.n_kv_heads // world * c.head_dim) % SHARD_COLUMN_ALIGN == 0
        self.kv_split = kv_split or world == 1
        group_size = c.n_heads // c.n_kv_heads
        self.kv_head0 = 0 if self.kv_split else rank * self.q_heads // group_size  # first KV head this rank reads
        self.kv_heads = c.n_kv_heads // world if self.kv_split else self.q_heads // group_size

        # ---- Q | K | V packed column-wise, one launch per run of equal types (Q4_K_M files
        # often keep attn_v in another type), their biases alike ----
        parts = []  # (bytes [K, rb], type, n_loc, bias or None)
        self.qkv_widths = []
        for name in ("attn_q", "attn_k", "attn_v"):
            split = name == "attn_q" or self.kv_split
            w = f.upload_shard(p + name + ".weight", "column", rank, world, self.dev) if split and world > 1 \
                else f.upload(p + name + ".weight", self.dev)
            K, N, t = f.matrix_shape(p + name + ".weight")
            n_loc = N // world if split else N
            bias = None
            b = f.tensor_info(p + name + ".bias")
            if b is not None and b.type == F.GGML_TYPE_F32:
                bt = f.upload(p + name + ".bias", self.dev).view(torch.float32).view(-1)
                bias = (bt[rank * n_loc:(rank + 1) * n_loc] if split else bt).contiguous()
            parts.append((w, t, n_loc, bias))
            self.qkv_widths.append(n_loc)
        self.qkv_mats = []  # (packed bytes, type, N, packed bias or None)
        i = 0
        while i < 3:
            j = i
            while j + 1 < 3 and parts[j + 1][1] == parts[i][1]:
                j += 1
            run = parts[i:j + 1]
            n = sum(r[2] for r in run)
            bias = None
            if any(r[3] is not None for r in run):
                bias = torch.cat([r[3] if r[3] is not None else torch.zeros(r[2], device=self.dev) for r in run])
            w = run[0][0] if len(run) == 1 else torch.cat([r[0] for r in run], dim=1).contiguous()
            self.qkv_mats.append((w, run[0][1], n, bias))
            i = j + 1

        # ---- o: row split ----
        self.o_type = f.matrix_shape(p + "attn_output.weight")[2]
        self.w_o = f.upload_shard(p + "attn_output.weight", "row", rank, world, self.dev) if world > 1 \
            else f.upload(p + "attn_output.weight", self.dev)

        # ---- FFN: gate | up packed column-wise, down row split ----
        self.ffn_loc = c.ffn // world
        gate = f.upload_shard(p + "ffn_gate.weight", "column", rank, world, self.dev) if world > 1 \
            else f.upload(p + "ffn_gate.weight", self.dev)
        up = f.upload_shard(p + "ffn_up.weight", "column", rank, world, self.dev) if world > 1 \
            else f.upload(p + "ffn_up.weight", self.dev)
        self.gu_type = self._same_type([f.matrix_shape(p + "ffn_gate.weight")[2],
                                        f.matrix_shape(p + "ffn_up.weight")[2]], "gate / up")
        self.w_gu = torch.cat([gate, up], dim=1).contiguous()
        self.down_type = f.matrix_shape(p + "ffn_down.weight")[2]
        self.w_down = f.upload_shard(p + "ffn_down.weight", "row", rank, world, self.dev) if world > 1 \
            else f.upload(p + "ffn_down.weight", self.dev)

        # norms (F32 vectors, replicated)
        self.attn_norm = f.upload(p + "attn_norm.weight", self.dev).view(torch.float32).view(-1)
        self.ffn_norm = f.upload(p + "ffn_norm.weight", self.dev).view(torch.float32).view(-1)

    @staticmethod
    def _same_type(types, what) -> int:
        if len(set(types)) != 1:
            raise ValueError(f"{what} weights have different types {types}; they are packed into one matrix")
        return types[0]

    # ---- matmul plumbing ----
    @staticmethod
    def _gemm_ok(t: int, K: int, N: int) -> bool:
        """Whether the tcgen05 GEMM takes a K x N matrix of type t."""
        return t in F.QUANTIZED and N % 256 == 0 and F.row_bytes(t, N) % 16 == 0 and K % 8 == 0

    def _mm(self, x: torch.Tensor, w: torch.Tensor, K: int, N: int, t: int, *, bias=None, residual=None,
            swiglu_input=False, prefill: bool, out_dtype=torch.float32) -> torch.Tensor:
        """x [T, K] (or [T, 2K] with swiglu_input) times W -> [T, N]: the fused GEMV (bias and
        residual in its epilogue) at decode; at prefill the tcgen05 GEMM when it takes the
        matrix (quantized, N whole 256-column tiles, rows a multiple of 16 bytes), else the
        GEMV over chunks of 32 tokens.  A SwiGLU input runs as its own pass first: read
        inside the GEMV it would be recomputed by every 256-column tile (measured on the 70B
        down projection: 48 us plain against 77 us fused at batch 1, 304 against 892 at 16)."""
        T = x.shape[0]
        if prefill and self._gemm_ok(t, K, N):
            a = x.to(torch.bfloat16).contiguous()
            if swiglu_input:
                a = swiglu_rows(a, K)
            return gemm_dequant(a, w, None, T, K, N, t, out_dtype=out_dtype, bias=bias,
                                residual=None if residual is None else residual.to(out_dtype).contiguous())
        xf = x.float().contiguous()
        if swiglu_input:
            xf = swiglu_rows(xf, K)
        out = torch.empty(T, N, device=x.device)
        for t0 in range(0, T, DECODE_MAX_TOKENS):
            t1 = min(T, t0 + DECODE_MAX_TOKENS)
            gemv_fused(xf[t0:t1], w, out[t0:t1], K, N, t, bias=bias,
                       residual=None if residual is None else residual[t0:t1].float().contiguous())
        return out if out_dtype == torch.float32 else out.to(out_dtype)

    def _reduce(self, y: torch.Tensor) -> torch.Tensor:
        if self.world > 1 and self.reduce:
            import torch.distributed as dist
            dist.all_reduce(y, group=self.group)
        return y

    # ---- the block's matmul steps ----
    def qkv(self, h: torch.Tensor, prefill: bool | None = None):
        """h [T, hidden] (normed) -> q [T, q_heads * hd], k, v [T, kv_heads * hd] of this
        rank's heads (biases added in the epilogue)."""
        prefill = h.shape[0] > DECODE_MAX_TOKENS if prefill is None else prefill
        ys = [self._mm(h, w, self.cfg.hidden, n, t, bias=b, prefill=prefill) for w, t, n, b in self.qkv_mats]
        y = ys[0] if len(ys) == 1 else torch.cat(ys, dim=1)
        q, k, v = torch.split(y, self.qkv_widths, dim=1)
        if not self.kv_split:  # replicated K / V: the heads this rank's queries read
            hd = self.cfg.head_dim
            s = slice(self.kv_head0 * hd, (self.kv_head0 + self.kv_heads) * hd)
            k, v = k[:, s], v[:, s]
        return q.contiguous(), k.contiguous(), v.contiguous()

    def attn_out(self, attn: torch.Tensor, residual: torch.Tensor, prefill: bool | None = None) -> torch.Tensor:
        """residual + attn Wo (cpp/src/fast_model.cpp:806-824); attn [T, q_heads * hd] of
        this rank's heads, residual fp32 [T, hidden]."""
        prefill = attn.shape[0] > DECODE_MAX_TOKENS if prefill is None else prefill
        res = residual.float().contiguous() if self.rank == 0 else None
        K = self.q_heads * self.cfg.head_dim
        y = self._mm(attn, self.w_o, K, self.cfg.hidden, self.o_type, residual=res, prefill=prefill)
        return self._reduce(y)

    def ffn(self, h: torch.Tensor, residual: torch.Tensor, prefill: bool | None = None) -> torch.Tensor:
        """residual + down(silu(h Wgate) * (h Wup)) (cpp/src/fast_model.cpp:906-998)."""
        prefill = h.shape[0] > DECODE_MAX_TOKENS if prefill is None else prefill
        c = self.cfg
        res = residual.float().contiguous() if self.rank == 0 else None
        gate_bytes = F.row_bytes(self.gu_type, self.ffn_loc)
        if (prefill and self._gemm_ok(self.gu_type, c.hidden, 2 * self.ffn_loc) and self.ffn_loc % 256 == 0
                and gate_bytes % 16 == 0):
            # gate | up and SwiGLU in one GEMM (the [T, 2I] intermediate never written)
            hs = gemm_swiglu(h.to(torch.bfloat16).contiguous(), self.w_gu, self.w_gu.view(-1)[gate_bytes:], None,
                             h.shape[0], c.hidden, self.ffn_loc, self.gu_type, row_bytes=2 * gate_bytes)
            y = self._mm(hs, self.w_down, self.ffn_loc, c.hidden, self.down_type, residual=res, prefill=True)
            return self._reduce(y)
        gu = self._mm(h, self.w_gu, c.hidden, 2 * self.ffn_loc, self.gu_type, prefill=prefill,
                      out_dtype=torch.bfloat16 if prefill else torch.float32)
        y = self._mm(gu, self.w_down, self.ffn_loc, c.hidden, self.down_type, residual=res,
                     swiglu_input=True, prefill=prefill)
        return self._reduce(y)

    def forward(self, x: torch.Tensor, attention, norm=None, prefill: bool | None = None) -> torch.Tensor:
        """The block on x [T, hidden] fp32: ``attention(q, k, v)`` is the engine's RoPE + KV
        cache + attention over this rank's heads, returning [T, q_heads * head_dim];
        ``norm(x, w, eps)`` defaults to the reference's RMSNorm."""
        norm = norm or rms_norm
        c = self.cfg
        q, k, v = self.qkv(norm(x, self.attn_norm, c.eps), prefill)
        x = self.attn_out(attention(q, k, v), x, prefill)
        return self.ffn(norm(x, self.ffn_norm, c.eps), x, prefill)
