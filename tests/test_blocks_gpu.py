"""The reference dispatcher's other block types on the device -- Q4_0, Q4_1, Q5_0, Q5_1,
Q2_K, Q3_K, Q5_K, Q8_K (cpp/src/dequant.cpp:23-245, :317-354, :407-425) -- through
vbq_dequantize and the generic GEMV kernel.

Dequantization is bit-exact against the reference's own outputs (committed golden
vectors) and the oracle pinned to it; the GEMV is within the path's 1e-3 max-norm bar of
the reference's sequential fp32 sums (small shapes) and of an fp64 product over the
bit-exact device dequantization (a 4096 x 14336 matrix), and bitwise deterministic."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import vibeblade_b200 as vb
from block_fill import BLOCK_VALUES, TYPES, edge_blocks, random_blocks
from conftest import bits_equal, load_golden, max_rel
from vibeblade_b200 import formats as F

pytestmark = pytest.mark.gpu

NAMES = [F.TYPE_NAMES[t].lower() for t in TYPES]


def bf16_rne(a: np.ndarray) -> np.ndarray:
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16).float().numpy()


@pytest.fixture(scope="module")
def golden():
    return load_golden("blocks")


@pytest.mark.parametrize("name", NAMES)
def test_dequant_golden_bitexact(cuda, golden, name):
    t = F.NAME_TO_TYPE[name.upper()]
    K, N = int(golden["K"]), int(golden["N"])
    w = torch.from_numpy(golden[f"{name}_w"]).to(cuda)
    assert bits_equal(vb.dequantize(w, K, N, t).cpu().numpy(), golden[f"{name}_deq"])
    gb = vb.dequantize(w, K, N, t, dtype=torch.bfloat16).float().cpu().numpy()
    assert bits_equal(gb, bf16_rne(golden[f"{name}_deq"]))
    wr = golden[f"{name}_random_w"]  # unconstrained bytes: inf / NaN scales
    got = vb.dequantize(torch.from_numpy(wr).to(cuda), wr.shape[0], N, t).cpu().numpy()
    assert bits_equal(got, golden[f"{name}_random_deq"])
    n = int(golden["ragged_n"])
    row = vb.dequantize_row(torch.from_numpy(golden[f"{name}_w"][0].copy()).to(cuda), None, n, t)
    assert row.shape == (n,)
    assert bits_equal(row.cpu().numpy(), golden[f"{name}_ragged_deq"])


@pytest.mark.parametrize("qtype", TYPES)
def test_dequant_random_vs_oracle(cuda, oracle, qtype):
    rng = np.random.default_rng(40 + qtype)
    for K, N in ((64, 4096), (5, 3 * BLOCK_VALUES[qtype])):
        for w in (random_blocks(qtype, K, N, rng), edge_blocks(qtype, K, N, rng)):
            got = vb.dequantize(torch.from_numpy(w).to(cuda), K, N, qtype).cpu().numpy()
            assert bits_equal(got, oracle.dequantize(w, K, N, qtype))
    for n in (1, 9, 33, BLOCK_VALUES[qtype] + 17):  # ragged single rows
        row = random_blocks(qtype, 1, n, rng)[0]
        got = vb.dequantize_row(torch.from_numpy(row).to(cuda), None, n, qtype).cpu().numpy()
        assert bits_equal(got, oracle.dequantize_row(row, n, qtype)), n


@pytest.mark.parametrize("name", NAMES)
def test_gemv_golden(cuda, golden, name):
    t = F.NAME_TO_TYPE[name.upper()]
    K, N = int(golden["K"]), int(golden["N"])
    x = torch.from_numpy(golden[f"{name}_x"]).to(cuda)
    y = vb.gemv_dequant(x, torch.from_numpy(golden[f"{name}_w"]).to(cuda), None, K, N, t)
    assert max_rel(y.cpu().numpy(), golden[f"{name}_gemv"]) <= 1e-3


@pytest.mark.parametrize("qtype", TYPES)
@pytest.mark.parametrize("batch", [1, 4, 7])
def test_gemv_vs_oracle(cuda, oracle, qtype, batch):
    """Random codes with N(0, 0.01) scales; widths of whole 256-column tiles and, for the
    32-value types, a width that ends inside a tile; batches across the kernel's groups of 4."""
    rng = np.random.default_rng(qtype * 10 + batch)
    shapes = [(512, 1024)] + ([(300, 96)] if BLOCK_VALUES[qtype] == 32 else [(300, 768)])
    for K, N in shapes:
        w = random_blocks(qtype, K, N, rng)
        x = rng.normal(0, 1, (batch, K)).astype(np.float32)
        wd = torch.from_numpy(w).to(cuda)
        y = vb.gemv_dequant(torch.from_numpy(x).to(cuda), wd, None, K, N, qtype).cpu().numpy()
        assert max_rel(y, oracle.gemv_dequant(x, w, K, N, qtype)) <= 1e-3
        y2 = vb.gemv_dequant(torch.from_numpy(x).to(cuda), wd, None, K, N, qtype).cpu().numpy()
        assert np.array_equal(y, y2)  # deterministic


@pytest.mark.parametrize("qtype", [F.GGML_TYPE_Q5_K, F.GGML_TYPE_Q4_0, F.GGML_TYPE_Q3_K])
def test_gemv_full_size_vs_fp64(cuda, qtype):
    """Config 2's 4096 x 14336 in a block type outside the path's three, batch 1 and 4,
    against an fp64 product of the device dequantization (itself bit-exact, above)."""
    K, N = 4096, 14336
    rng = np.random.default_rng(qtype)
    wd = torch.from_numpy(random_blocks(qtype, K, N, rng, std=2e-4)).to(cuda)
    deq = vb.dequantize(wd, K, N, qtype).double()
    for batch in (1, 4):
        x = torch.from_numpy(rng.normal(0, 1, (batch, K)).astype(np.float32)).to(cuda)
        y = vb.gemv_dequant(x, wd, None, K, N, qtype)
        ref = x.double() @ deq
        err = float((y.double() - ref).abs().max() / ref.abs().max())
        assert err <= 1e-3, err


@pytest.mark.parametrize("qtype", [F.GGML_TYPE_Q4_1, F.GGML_TYPE_Q8_K])
def test_gemv_fused_epilogue(cuda, qtype):
    """Bias and residual added in the generic kernel's epilogue: the same as adding them
    after the plain GEMV."""
    K, N, batch = 256, 512, 3
    rng = np.random.default_rng(qtype + 77)
    wd = torch.from_numpy(random_blocks(qtype, K, N, rng)).to(cuda)
    x = torch.from_numpy(rng.normal(0, 1, (batch, K)).astype(np.float32)).to(cuda)
    bias = torch.from_numpy(rng.normal(0, 1, N).astype(np.float32)).to(cuda)
    res = torch.from_numpy(rng.normal(0, 1, (batch, N)).astype(np.float32)).to(cuda)
    plain = vb.gemv_dequant(x, wd, None, K, N, qtype)
    fused = vb.gemv_fused(x, wd, None, K, N, qtype, bias=bias, residual=res)
    assert torch.equal(fused, plain + bias + res)


def test_gguf_upload_and_shards(cuda, tmp_path):
    """GGUF tensors of these types arrive as the file's bytes (whole and as tensor-parallel
    column / row shards), and the GEMV reads them like the uploaded matrix."""
    import gguf_files as G
    from vibeblade_b200 import tp
    from vibeblade_b200.gguf import GGUFFile
    rng = np.random.default_rng(9)
    specs = [("a.weight", 512, 2048, F.GGML_TYPE_Q5_K), ("b.weight", 1024, 512, F.GGML_TYPE_Q4_0),
             ("c.weight", 256, 1024, F.GGML_TYPE_Q3_K), ("d.weight", 512, 512, F.GGML_TYPE_Q8_K)]
    ws = {name: random_blocks(t, K, N, rng) for name, K, N, t in specs}
    path = G.write(tmp_path / "m.gguf", [("general.architecture", G.STRING, "llama")],
                   [G.weight_tensor(name, ws[name], K, N, t) for name, K, N, t in specs])
    with GGUFFile(path) as f:
        for name, K, N, t in specs:
            assert f.matrix_shape(name) == (K, N, t)
            w = f.upload(name, cuda)
            whole = torch.from_numpy(ws[name]).to(cuda)
            assert torch.equal(w, whole)
            x = torch.from_numpy(rng.normal(0, 1, (2, K)).astype(np.float32)).to(cuda)
            assert torch.equal(vb.gemv_dequant(x, w, None, K, N, t), vb.gemv_dequant(x, whole, None, K, N, t))
            for kind in ("column", "row"):
                for r in range(2):
                    assert torch.equal(f.upload_shard(name, kind, r, 2, cuda),
                                       tp.shard(whole, K, N, t, kind, r, 2))


def test_tp_linear_emulated(cuda):
    """A Q5_K layer split over 2 ranks (emulated on one GPU): column shards concatenate and
    row shards sum to the unsplit GEMV, at decode and at prefill (where these types run
    the generic GEMV over all rows instead of the tensor-core GEMM)."""
    from vibeblade_b200 import tp
    K, N, t = 1024, 2048, F.GGML_TYPE_Q5_K
    rng = np.random.default_rng(11)
    w = torch.from_numpy(random_blocks(t, K, N, rng, std=1e-3)).to(cuda)
    x = torch.from_numpy(rng.normal(0, 1, (5, K)).astype(np.float32)).to(cuda)
    full = vb.gemv_dequant(x, w, None, K, N, t)
    a = x.to(torch.bfloat16)
    full_a = vb.gemv_dequant(a.float(), w, None, K, N, t)
    cols = [tp.TPLinear(w, K, N, t, "column", r, 2, cuda) for r in range(2)]
    # a shard's columns are summed over the same rows as the whole matrix's (split-K
    # order may differ with the shard's width)
    for got, want in ((torch.cat([c.decode(x) for c in cols], dim=1), full),
                      (torch.cat([c.prefill(a) for c in cols], dim=1), full_a)):
        assert float((got - want).abs().max() / want.abs().max()) <= 1e-5
    rows = [tp.TPLinear(w, K, N, t, "row", r, 2, cuda) for r in range(2)]
    part = sum(r.decode(x[:, i * K // 2:(i + 1) * K // 2].contiguous()) for i, r in enumerate(rows))
    assert float((part - full).abs().max() / full.abs().max()) <= 1e-5
    pre = sum(r.prefill(a[:, i * K // 2:(i + 1) * K // 2]) for i, r in enumerate(rows))
    assert float((pre - full_a).abs().max() / full_a.abs().max()) <= 1e-5


def test_gguf_dequant_row(cuda, oracle, tmp_path):
    """GGUFFile.dequant_row (the reference's VibeBladeFast.dequant_row debug binding,
    cpp/src/bindings.cpp:407-436) on every type it takes: one row, a prefix of a row, and a
    count running on into the next row, bit-exact against the oracle's dequantize_row of
    the same bytes."""
    import gguf_files as G
    from vibeblade_b200.gguf import GGUFFile
    from vibeblade_b200.quantize import synthetic_weights
    rng = np.random.default_rng(21)
    K, N = 3, 512
    ws = {F.GGML_TYPE_Q4_0: random_blocks(F.GGML_TYPE_Q4_0, K, N, rng),
          F.GGML_TYPE_Q5_0: random_blocks(F.GGML_TYPE_Q5_0, K, N, rng),
          F.GGML_TYPE_Q5_K: random_blocks(F.GGML_TYPE_Q5_K, K, N, rng),
          F.GGML_TYPE_F32: rng.normal(0, 1, (K, N)).astype(np.float32).view(np.uint8),
          F.GGML_TYPE_F16: rng.normal(0, 1, (K, N)).astype(np.float16).view(np.uint8)}
    for t in (F.GGML_TYPE_Q4_K, F.GGML_TYPE_Q6_K, F.GGML_TYPE_Q8_0):
        ws[t] = synthetic_weights(K, N, t, seed=t).numpy()
    path = G.write(tmp_path / "r.gguf", [],
                   [G.weight_tensor(F.TYPE_NAMES[t], w, K, N, t) for t, w in ws.items()])
    with GGUFFile(path) as f:
        for t, w in ws.items():
            flat = np.ascontiguousarray(w).view(np.uint8).reshape(-1)
            rb = F.row_bytes(t, N)
            for row, n in ((1, 0), (2, 100), (0, 2 * N)):
                got = f.dequant_row(F.TYPE_NAMES[t], row, n, device=cuda)
                nn = n if n > 0 else N
                want = oracle.dequantize_row(flat[row * rb:], nn, t)
                assert got.shape == (nn,) and bits_equal(got, want), (t, row, n)


@pytest.mark.parametrize("qtype", [F.GGML_TYPE_Q5_K, F.GGML_TYPE_Q4_0])
def test_gemv_swiglu_input(cuda, qtype):
    """The fused SwiGLU input (x = silu(gate) * up of a packed [B, 2K] buffer) gives the
    same bits as a SwiGLU pass followed by the plain GEMV."""
    from vibeblade_b200 import tp
    K, N, batch = 512, 1024, 5
    rng = np.random.default_rng(qtype + 3)
    wd = torch.from_numpy(random_blocks(qtype, K, N, rng)).to(cuda)
    gu = torch.from_numpy(rng.normal(0, 2, (batch, 2 * K)).astype(np.float32)).to(cuda)
    fused = vb.gemv_fused(gu, wd, None, K, N, qtype, swiglu_input=True)
    plain = vb.gemv_dequant(tp.swiglu_rows(gu, K), wd, None, K, N, qtype)
    assert torch.equal(fused, plain)


def test_gemv_long_rows_fall_back(cuda, oracle):
    """A K-slice whose activations overflow the staged kernel's shared memory (very long
    rows at batch 4, a type the tensor-core kernels do not take) runs on the generic
    kernel instead, with the same bar."""
    K, N, batch, t = 120000, 256, 4, F.GGML_TYPE_Q2_K
    rng = np.random.default_rng(8)
    w = random_blocks(t, K, N, rng, std=1e-3)
    x = rng.normal(0, 1, (batch, K)).astype(np.float32)
    y = vb.gemv_dequant(torch.from_numpy(x).to(cuda), torch.from_numpy(w).to(cuda), None, K, N, t)
    assert max_rel(y.cpu().numpy(), oracle.gemv_dequant(x, w, K, N, t)) <= 1e-3


def _outlier_rows(rng, batch, K, frac=0.01, lo=100.0, hi=1000.0):
    """N(0, 1) activations with `frac` of each row's channels scaled 100-1000x (random sign)
    and one at the last row of the first 32-row slice, like real hidden states."""
    x = rng.normal(0, 1, (batch, K)).astype(np.float32)
    n = max(1, int(frac * K))
    for b in range(batch):
        idx = rng.choice(K, n, replace=False)
        x[b, idx] *= (rng.uniform(lo, hi, n) * rng.choice([-1.0, 1.0], n)).astype(np.float32)
        x[b, 31] = np.float32(hi)
    return x


def _columns_ok(y, ref, what):
    """1e-3 of each row's largest output, and 1e-3 relative on every output >= 1e-2 of it."""
    y, ref = np.asarray(y, np.float64), np.asarray(ref, np.float64)
    mx = np.abs(ref).max(axis=1, keepdims=True)
    err = np.abs(y - ref)
    assert (err / mx).max() <= 1e-3, f"{what}: max-norm {(err / mx).max():.3g}"
    big = np.abs(ref) >= 1e-2 * mx
    assert (err[big] / np.abs(ref[big])).max() <= 1e-3, f"{what}: per-column"


@pytest.mark.parametrize("t", [F.GGML_TYPE_Q5_K, F.GGML_TYPE_Q4_0, F.GGML_TYPE_Q4_1, F.GGML_TYPE_Q5_0,
                               F.GGML_TYPE_Q5_1])
@pytest.mark.parametrize("K,N", [(4096, 14336), (14336, 4096)])
@pytest.mark.parametrize("batch", [1, 2, 4, 16])
def test_tensor_core_gemv_outliers(cuda, oracle, t, K, N, batch):
    """Decode batches of these types run on the integer tensor cores: Q5_K on the Q4_K
    kernel's form (fifth bits merged into the A fragments, codes 0..31 in u8), Q4_0 / Q4_1 /
    Q5_0 / Q5_1 on the Q8_0 kernel's (nibbles as u8 codes, fifth bits from qh, the -8 / -16
    offsets and the + m terms summed apart).  Outlier activations, per-column bar, against
    the fp64 product of the bit-exact device dequantization and the reference's sequential
    fp32 sums; the device status stays clean and repeats are bit-identical."""
    rng = np.random.default_rng(K + batch + t)
    wh = random_blocks(t, K, N, rng, std=2e-4)
    w = torch.from_numpy(wh).to(cuda)
    x = _outlier_rows(rng, batch, K)
    xd = torch.from_numpy(x).to(cuda)
    y = vb.gemv_dequant(xd, w, None, K, N, t)
    assert torch.equal(y, vb.gemv_dequant(xd, w, None, K, N, t))
    assert vb.device_status() == 0
    deq = vb.dequantize(w, K, N, t).double()
    ref64 = (xd.double() @ deq).cpu().numpy()
    del deq
    _columns_ok(y.cpu().numpy(), ref64, "fp64")
    if batch <= 4:
        _columns_ok(y.cpu().numpy(), oracle.gemv_dequant(x, wh, K, N, t), "oracle")
