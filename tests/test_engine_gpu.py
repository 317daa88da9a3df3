"""Engine integration: a transformer block loaded from a GGUF file and run through
vibeblade_b200.engine.DeviceLayer (every matmul of the block on the device kernels, the
element-wise steps fused in) against the reference's own block.

Golden vectors: tests/golden/layer_llama.npz, written by tests/golden/make_layer_golden.py
from the reference's forward_token (vibeblade/transformer.py:232-325) on four positions
with a KV cache, over the bit-exact dequantization of the fixture's Q4_K / Q6_K / Q8_0
matrices.  RoPE and attention -- the engine's part, outside the matmul path -- are restated
here in torch after vibeblade/transformer.py:73-174.  Bars: 1e-3 (fp32 decode GEMVs) and
2e-2 (bf16 prefill GEMMs), max-norm relative."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import gguf_files as G
from conftest import load_golden
from vibeblade_b200.engine import DeviceLayer, LayerConfig
from vibeblade_b200.gguf import GGUFFile

pytestmark = pytest.mark.gpu

NAMES = ["attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"]


@pytest.fixture(scope="module")
def golden(tmp_path_factory):
    g = load_golden("layer_llama")
    tensors = []
    for n in NAMES:
        w = g[f"{n}_bytes"]
        K = w.shape[0]
        t = int(g[f"{n}_type"])
        from vibeblade_b200 import formats as F
        N = w.shape[1] // F.BLOCK_BYTES[t] * F.BLOCK_VALUES[t]
        tensors.append(G.weight_tensor(f"blk.0.{n}.weight", w, K, N, t))
    for n in ("attn_norm", "ffn_norm"):
        tensors.append((f"blk.0.{n}.weight", (int(g["hidden"]),), 0, g[n].astype(np.float32).tobytes()))
    kv = [("general.architecture", G.STRING, "llama"), ("llama.embedding_length", G.U32, int(g["hidden"])),
          ("llama.attention.head_count", G.U32, int(g["n_heads"])),
          ("llama.attention.head_count_kv", G.U32, int(g["n_kv_heads"])),
          ("llama.feed_forward_length", G.U32, int(g["ffn"])),
          ("llama.attention.layer_norm_rms_epsilon", G.F32, float(g["eps"]))]
    path = G.write(tmp_path_factory.mktemp("layer") / "model.gguf", kv, tensors)
    return path, g


def _rope_tables(head_dim, n, dev):
    # build_rope_cache (vibeblade/transformer.py:102-112), float32 throughout
    inv = 1.0 / (10000.0 ** (np.arange(0, head_dim, 2, dtype=np.float32) / head_dim))
    fr = np.outer(np.arange(n, dtype=np.float32), inv)
    return torch.from_numpy(np.cos(fr).astype(np.float32)).to(dev), torch.from_numpy(np.sin(fr).astype(np.float32)).to(dev)


class Attention:
    """RoPE (halves rotated, transformer.py:73-99) + KV cache + grouped-query softmax
    attention (transformer.py:115-174) over a rank's query heads and their KV heads."""

    def __init__(self, head_dim, cos, sin):
        self.hd, self.cos, self.sin = head_dim, cos, sin
        self.k = self.v = None

    def rope(self, x, pos0):
        T, n = x.shape[0], x.shape[1] // self.hd
        x = x.view(T, n, self.hd)
        c = self.cos[pos0:pos0 + T].unsqueeze(1)
        s = self.sin[pos0:pos0 + T].unsqueeze(1)
        h = self.hd // 2
        x0, x1 = x[..., :h], x[..., h:]
        return torch.cat([x0 * c - x1 * s, x1 * c + x0 * s], dim=-1).view(T, n * self.hd)

    def __call__(self, q, k, v):
        pos0 = 0 if self.k is None else self.k.shape[0]
        q, k = self.rope(q, pos0), self.rope(k, pos0)
        self.k = k if self.k is None else torch.cat([self.k, k])
        self.v = v if self.v is None else torch.cat([self.v, v])
        T, S = q.shape[0], self.k.shape[0]
        nq, nkv = q.shape[1] // self.hd, self.k.shape[1] // self.hd
        qh = q.view(T, nq, self.hd).transpose(0, 1)
        kh = self.k.view(S, nkv, self.hd).transpose(0, 1).repeat_interleave(nq // nkv, dim=0)
        vh = self.v.view(S, nkv, self.hd).transpose(0, 1).repeat_interleave(nq // nkv, dim=0)
        sc = qh @ kh.transpose(1, 2) * (1.0 / np.sqrt(float(self.hd)))
        mask = torch.full((T, S), float("-inf"), device=q.device)
        for i in range(T):
            mask[i, :S - T + i + 1] = 0.0
        p = torch.softmax(sc + mask, dim=-1)
        return (p @ vh).transpose(0, 1).reshape(T, nq * self.hd)


def _rel(a, b):
    b = torch.as_tensor(b, device=a.device)
    return ((a.double() - b.double()).abs().max() / b.double().abs().max()).item()


def test_decode_matches_reference_forward_token(cuda, golden):
    path, g = golden
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        with GGUFFile(path) as f:
            layer = DeviceLayer(f, 0, cuda)
        cfg = layer.cfg
        assert (cfg.hidden, cfg.n_heads, cfg.n_kv_heads, cfg.ffn) == (512, 8, 4, 1024)
        cos, sin = _rope_tables(cfg.head_dim, 64, cuda)
        att = Attention(cfg.head_dim, cos, sin)
        x = torch.from_numpy(g["x"]).to(cuda)
        for pos in range(x.shape[0]):
            y = layer.forward(x[pos:pos + 1], att, prefill=False)
            assert _rel(y[0], g["y"][pos]) <= 1e-3, pos
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def test_prefill_matches_reference_forward_token(cuda, golden):
    """All four positions at once through the prefill path (tcgen05 GEMM where the matrix
    fits it, bf16 activations), causal attention; equal to the reference's position-by-
    position decode within the bf16 bar."""
    path, g = golden
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        with GGUFFile(path) as f:
            layer = DeviceLayer(f, 0, cuda)
        cos, sin = _rope_tables(layer.cfg.head_dim, 64, cuda)
        x = torch.from_numpy(g["x"]).to(cuda)
        y = layer.forward(x, Attention(layer.cfg.head_dim, cos, sin), prefill=True)
        assert _rel(y, g["y"]) <= 2e-2
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def test_tensor_parallel_two_ranks_emulated(cuda, golden):
    """Two ranks' shards read from the file (Q and gate / up by columns, o and down by rows,
    K / V replicated since their 128-column shards are not whole tiles), each rank attending
    over its own heads; the partial sums added (the all-reduce) give the one-rank result."""
    path, g = golden
    with GGUFFile(path) as f:
        one = DeviceLayer(f, 0, cuda)
        ranks = [DeviceLayer(f, 0, cuda, rank=r, world=2, reduce=False) for r in range(2)]
    assert not ranks[0].kv_split and ranks[1].kv_head0 == 2
    cfg = one.cfg
    cos, sin = _rope_tables(cfg.head_dim, 64, cuda)
    x = torch.from_numpy(g["x"]).to(cuda)
    from vibeblade_b200.engine import rms_norm
    for prefill in (False, True):
        ref = one.forward(x, Attention(cfg.head_dim, cos, sin), prefill=prefill)
        atts = [Attention(cfg.head_dim, cos, sin) for _ in ranks]
        h = rms_norm(x, one.attn_norm, cfg.eps)
        x1 = sum(L.attn_out(a(*L.qkv(h, prefill)), x, prefill) for L, a in zip(ranks, atts))
        h2 = rms_norm(x1, one.ffn_norm, cfg.eps)
        y = sum(L.ffn(h2, x1, prefill) for L in ranks)
        assert _rel(y, ref) <= (2e-2 if prefill else 1e-4)
