"""MoE on the GPU: routing, grouped dequant-GEMM over expert slabs, and the full SwiGLU
MoE FFN, against the reference's own MoE output (golden) and the CPU restatement.

Tolerance: the north star's 2e-2 max-norm relative error for the bf16 tensor-core path
(activations and the SwiGLU product enter the MMAs as bf16, fp32 accumulation)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import vibeblade_b200 as vb
from conftest import load_golden, max_rel
from oracle.moe_oracle import moe_ffn as oracle_moe_ffn
from oracle.moe_oracle import route as oracle_route
from vibeblade_b200 import formats as F
from vibeblade_b200.quantize import quantize, synthetic_weights

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _slabs(rng, E, K, N, qtype):
    qs = [quantize(rng.normal(0, 0.02, (K, N)).astype(np.float32), qtype).numpy().reshape(-1)
          for _ in range(E)]
    return np.concatenate(qs)


def _dense(oracle, slabs, E, K, N, qtype):
    s = slabs.reshape(E, -1)
    return np.stack([oracle.dequantize(s[e], K, N, qtype) for e in range(E)])


def test_route_vs_oracle(cuda):
    rng = np.random.default_rng(7)
    lg = rng.normal(0, 1, (1000, 8)).astype(np.float32)
    lg[0] = [100, 50, -100, 0, 0, 0, 0, 0]        # clipped
    lg[1] = 1.0                                     # all tied
    lg[2, :] = -1.0
    lg[2, 3] = lg[2, 5] = 2.0                       # tie between two winners
    for k in (1, 2, 4, 8):
        idx, w = vb.moe_route(torch.from_numpy(lg).to(cuda), k)
        ri, rw = oracle_route(lg, k)
        assert np.array_equal(idx.cpu().numpy(), ri)
        np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=2e-6, atol=1e-7)


def _stable_sort_ref(idx: np.ndarray, E: int):
    """Stable counting sort of the flattened entries by expert (entries outside 0..E-1
    skipped): the row layout the device MoE uses."""
    flat = idx.reshape(-1)
    k = idx.shape[1]
    seg = np.zeros(E + 1, np.int32)
    for e in range(E):
        seg[e + 1] = seg[e] + int(np.sum(flat == e))
    pos = np.full(flat.size, -1, np.int32)
    tok = np.full(flat.size, -1, np.int32)
    nxt = seg[:-1].copy()
    for j, e in enumerate(flat):
        if 0 <= e < E:
            pos[j] = nxt[e]
            tok[nxt[e]] = j // k
            nxt[e] += 1
    return seg, pos, tok


@pytest.mark.parametrize("T,E,k", [(1, 8, 1), (33, 8, 2), (1000, 8, 2), (4096, 8, 2), (777, 64, 4),
                                   (300, 200, 8), (50, 1000, 2)])
def test_moe_sort_is_stable_counting_sort(cuda, T, E, k):
    """vbq_moe_sort (one CTA, 32 warps on contiguous chunks; the single-warp form above
    384 experts) against a plain stable counting sort, with skipped (out-of-range) entries
    and sizes that do not divide evenly among the warps."""
    rng = np.random.default_rng(T * 7 + E + k)
    idx = rng.integers(0, E, (T, k)).astype(np.int32)
    idx.reshape(-1)[::13] = -1
    idx.reshape(-1)[5::29] = E + 3
    seg, pos, tok = vb.moe_sort(torch.from_numpy(idx).to(cuda), E)
    rseg, rpos, rtok = _stable_sort_ref(idx, E)
    assert np.array_equal(seg.cpu().numpy(), rseg)
    assert np.array_equal(pos.cpu().numpy(), rpos)
    n = int(rseg[-1])
    assert np.array_equal(tok.cpu().numpy()[:n], rtok[:n])


def test_moe_ffn_matches_reference_golden(cuda):
    g = load_golden("moe_q4_k")
    T, H, I, E, k, t = (int(g[n]) for n in ("T", "H", "I", "E", "topk", "type"))
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    out = vb.moe_ffn(dev(g["x"]), dev(g["logits"]), dev(g["gate"]), dev(g["up"]), dev(g["down"]),
                     I, t, topk=k)
    torch.cuda.synchronize()
    assert vb.device_status() == 0
    assert max_rel(out.cpu().numpy(), g["out"]) <= TOL


@pytest.mark.parametrize("qtype,K,N", [(F.GGML_TYPE_Q4_K, 256, 512), (F.GGML_TYPE_Q8_0, 320, 256),
                                       (F.GGML_TYPE_Q6_K, 128, 2048)])
def test_gemm_grouped_vs_oracle(cuda, oracle, qtype, K, N):
    rng = np.random.default_rng(K + N + qtype)
    E = 5
    slabs = _slabs(rng, E, K, N, qtype)
    # ragged segments: empty, one row, a tile and a bit, several tiles, and rows after
    # the last segment that no segment owns
    sizes = [0, 1, 600, 130, 1100]
    seg = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int32)
    rows = int(seg[-1]) + 7
    a = torch.from_numpy(rng.normal(0, 1, (rows, K)).astype(np.float32)).to(torch.bfloat16)
    out = torch.full((rows, N), 123.0, dtype=torch.float32, device=cuda)
    vb.gemm_grouped(a.to(cuda), torch.from_numpy(slabs).to(cuda), torch.from_numpy(seg).to(cuda),
                    K, N, qtype, out=out)
    torch.cuda.synchronize()
    assert vb.device_status() == 0
    c = out.cpu().numpy()
    af = a.float().numpy()
    sl = slabs.reshape(E, -1)
    for e in range(E):
        lo, hi = int(seg[e]), int(seg[e + 1])
        if hi > lo:
            ref = oracle.gemm_f64(af[lo:hi], sl[e], hi - lo, K, N, qtype)
            assert max_rel(c[lo:hi], ref) <= TOL, e
    assert np.all(c[int(seg[-1]):] == 123.0)  # rows outside every segment untouched


@pytest.mark.parametrize("qtype,T,H,I,E,k", [(F.GGML_TYPE_Q4_K, 300, 512, 768, 6, 2),
                                             (F.GGML_TYPE_Q8_0, 129, 256, 512, 4, 3),
                                             (F.GGML_TYPE_Q6_K, 40, 2048, 2048, 3, 1)])
def test_moe_ffn_vs_oracle(cuda, oracle, qtype, T, H, I, E, k):
    rng = np.random.default_rng(T + H + I)
    wg, wu, wd = _slabs(rng, E, H, I, qtype), _slabs(rng, E, H, I, qtype), _slabs(rng, E, I, H, qtype)
    x = rng.normal(0, 1, (T, H)).astype(np.float32)
    lg = rng.normal(0, 1, (T, E)).astype(np.float32)
    dev = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    out = vb.moe_ffn(dev(x), dev(lg), dev(wg), dev(wu), dev(wd), I, qtype, topk=k)
    out2 = vb.moe_ffn(dev(x), dev(lg), dev(wg), dev(wu), dev(wd), I, qtype, topk=k)
    torch.cuda.synchronize()
    assert vb.device_status() == 0
    assert torch.equal(out, out2)  # deterministic
    ref = oracle_moe_ffn(x, lg, _dense(oracle, wg, E, H, I, qtype), _dense(oracle, wu, E, H, I, qtype),
                         _dense(oracle, wd, E, I, H, qtype), k, "fp32")
    assert max_rel(out.cpu().numpy(), ref) <= TOL


def test_moe_ffn_config4_sampled_tokens(cuda):
    """BASELINE config 4 (8 experts, top-2, hidden 4096, expert intermediate 14336, Q4_K,
    4096 tokens): full-size device run; 12 sampled tokens recomputed with torch fp32
    matmuls over the bit-exact device dequantization of their experts."""
    T, H, I, E, k = 4096, 4096, 14336, 8, 2
    qt = F.GGML_TYPE_Q4_K
    nb_gu, nb_d = F.matrix_nbytes(qt, H, I), F.matrix_nbytes(qt, I, H)
    wg = torch.empty(E * nb_gu, dtype=torch.uint8, device=cuda)
    wu = torch.empty(E * nb_gu, dtype=torch.uint8, device=cuda)
    wd = torch.empty(E * nb_d, dtype=torch.uint8, device=cuda)
    for e in range(E):
        wg[e * nb_gu:(e + 1) * nb_gu] = synthetic_weights(H, I, qt, seed=10 + e, device=cuda).reshape(-1)
        wu[e * nb_gu:(e + 1) * nb_gu] = synthetic_weights(H, I, qt, seed=20 + e, device=cuda).reshape(-1)
        wd[e * nb_d:(e + 1) * nb_d] = synthetic_weights(I, H, qt, seed=30 + e, device=cuda).reshape(-1)
    gen = torch.Generator(device=cuda).manual_seed(3)
    x = torch.randn(T, H, generator=gen, device=cuda)
    lg = torch.randn(T, E, generator=gen, device=cuda)
    out = vb.moe_ffn(x, lg, wg, wu, wd, I, qt, topk=k)
    out2 = vb.moe_ffn(x, lg, wg, wu, wd, I, qt, topk=k)
    idx, w = vb.moe_route(lg, k)
    torch.cuda.synchronize()
    assert vb.device_status() == 0
    assert torch.equal(out, out2)
    toks = torch.tensor([0, 1, 7, 100, 511, 1024, 2047, 2048, 3000, 4000, 4094, 4095], device=cuda)
    xs = x[toks].to(torch.bfloat16).float()
    ref = torch.zeros(len(toks), H, device=cuda)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for e in range(E):
            sel = (idx[toks] == e)
            if not sel.any():
                continue
            rows = sel.any(dim=1).nonzero().flatten()
            we = (w[toks] * sel).sum(dim=1)[rows]
            G = vb.dequantize(wg[e * nb_gu:(e + 1) * nb_gu], H, I, qt)
            U = vb.dequantize(wu[e * nb_gu:(e + 1) * nb_gu], H, I, qt)
            g = (xs[rows] @ G).clamp(-65504, 65504)
            u = (xs[rows] @ U).clamp(-65504, 65504)
            del G, U
            h = (torch.nn.functional.silu(g) * u).to(torch.bfloat16).float()
            D = vb.dequantize(wd[e * nb_d:(e + 1) * nb_d], I, H, qt)
            ref[rows] += we[:, None] * (h @ D)
            del D
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    err = ((out[toks] - ref).abs().max() / ref.abs().max()).item()
    assert err <= TOL
