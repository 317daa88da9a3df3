"""Device fused dequant-GEMV vs the reference's gemv_dequant.

Tolerance: max-norm relative error <= 1e-3 (fp32 outputs), the bound the north star states.
Small cases compare against the golden vectors and the oracle (the reference's own
sequential fp32 accumulation); BASELINE-size cases compare against an fp64 product of
the bit-exact device dequantization and check size-independent properties (linearity
in x, batch-row independence, determinism)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import vibeblade_b200 as vb
from conftest import load_golden, max_rel
from vibeblade_b200 import formats as F
from vibeblade_b200.quantize import quantize, synthetic_weights

pytestmark = pytest.mark.gpu

TOL = 1e-3
TYPES = [F.GGML_TYPE_Q4_K, F.GGML_TYPE_Q6_K, F.GGML_TYPE_Q8_0]


@pytest.mark.parametrize("name", ["q4_k", "q6_k", "q8_0"])
def test_gemv_golden(cuda, name):
    g = load_golden(name)
    K, N, t = int(g["K"]), int(g["N"]), int(g["type"])
    fin = np.isfinite(g["gemv_f64"]).all(axis=0)
    x = torch.from_numpy(g["x"]).to(cuda)
    w = torch.from_numpy(g["w"]).to(cuda)
    y = vb.gemv_dequant(x, w, None, K, N, t).cpu().numpy()
    ref = g["gemv"] if "gemv" in g else g["gemv_f64"]
    assert fin.all()
    assert max_rel(y, ref) <= TOL


@pytest.mark.parametrize("qtype", TYPES)
@pytest.mark.parametrize("batch", [1, 2, 3, 4, 5, 8, 11, 16])
def test_gemv_vs_oracle_small(cuda, oracle, qtype, batch):
    K, N = 300, 1024
    rng = np.random.default_rng(batch * 31 + qtype)
    w = quantize(rng.normal(0, 0.02, (K, N)).astype(np.float32), qtype).numpy()
    x = rng.normal(0, 1, (batch, K)).astype(np.float32)
    ref = oracle.gemv_dequant(x, w, K, N, qtype)
    y = vb.gemv_dequant(torch.from_numpy(x).to(cuda), torch.from_numpy(w).to(cuda), None, K, N,
                        qtype).cpu().numpy()
    assert y.shape == (batch, N)
    assert max_rel(y, ref) <= TOL


@pytest.mark.parametrize("qtype", TYPES)
@pytest.mark.parametrize("K", [1, 63, 64, 65, 1000])
def test_gemv_ragged_k(cuda, oracle, qtype, K):
    N = 512
    rng = np.random.default_rng(K + qtype)
    w = quantize(rng.normal(0, 0.5, (K, N)).astype(np.float32), qtype).numpy()
    x = rng.normal(0, 1, (1, K)).astype(np.float32)
    ref = oracle.gemv_dequant(x, w, K, N, qtype)
    y = vb.gemv_dequant(torch.from_numpy(x).to(cuda), torch.from_numpy(w).to(cuda), None, K, N,
                        qtype).cpu().numpy()
    assert max_rel(y, ref) <= TOL


@pytest.mark.parametrize("qtype", [F.GGML_TYPE_Q4_K, F.GGML_TYPE_Q8_0])
@pytest.mark.parametrize("K,batch", [(63, 8), (65, 16), (1000, 13), (1000, 16), (300, 9)])
def test_gemv_batch_routing_ragged_k(cuda, oracle, qtype, K, batch):
    """Batches 5-16 take the one-pass kernel when x rows are 16-byte aligned (K % 4 == 0)
    and groups of 4 otherwise; every route matches the reference."""
    N = 768
    rng = np.random.default_rng(K * 17 + batch + qtype)
    w = quantize(rng.normal(0, 0.3, (K, N)).astype(np.float32), qtype).numpy()
    x = rng.normal(0, 1, (batch, K)).astype(np.float32)
    ref = oracle.gemv_dequant(x, w, K, N, qtype)
    y = vb.gemv_dequant(torch.from_numpy(x).to(cuda), torch.from_numpy(w).to(cuda), None, K, N,
                        qtype).cpu().numpy()
    assert max_rel(y, ref) <= TOL


@pytest.mark.parametrize("batch", [12, 16])
def test_gemv_misaligned_x_view(cuda, batch):
    """x as a view starting 4 bytes into its buffer: not 16-byte aligned, so batch 9-16
    cannot use the TMA read of x and runs in groups of 4; same result as an aligned copy."""
    K, N, t = 4096, 4096, F.GGML_TYPE_Q4_K
    w = synthetic_weights(K, N, t, seed=3, device=cuda)
    g = torch.Generator(device=cuda).manual_seed(5)
    buf = torch.randn(batch * K + 1, generator=g, device=cuda)
    x_view = buf[1:].view(batch, K)
    assert x_view.data_ptr() % 16 != 0
    y_view = vb.gemv_dequant(x_view, w, None, K, N, t)
    y_copy = vb.gemv_dequant(x_view.clone(), w, None, K, N, t)
    assert ((y_view - y_copy).abs().max() / y_copy.abs().max()).item() <= 1e-5
    assert vb.device_status() == 0


@pytest.mark.parametrize("qtype", [F.GGML_TYPE_Q4_K, F.GGML_TYPE_Q8_0])
def test_gemv_k_past_integer_cap(cuda, qtype):
    """K above the integer-MMA kernels' cap (their s32 sums must stay exact) runs on the
    fp32 kernel with caller scratch; same bar against the fp64 product."""
    K, N, B = 3 * 65536 + 2048, 512, 2
    w = synthetic_weights(K, N, qtype, seed=9, device=cuda)
    g = torch.Generator(device=cuda).manual_seed(10)
    x = torch.randn(B, K, generator=g, device=cuda)
    assert vb.gemv_scratch_bytes(K, N, qtype, B) > 0
    y = vb.gemv_dequant(x, w, None, K, N, qtype)
    ref = x.double() @ vb.dequantize(w, K, N, qtype).double()
    assert ((y.double() - ref).abs().max() / ref.abs().max()).item() <= TOL
    assert vb.device_status() == 0


@pytest.mark.parametrize("qtype", TYPES)
@pytest.mark.parametrize("batch", [17, 24, 32])
def test_gemv_batch_above_16(cuda, qtype, batch):
    """Batches 17..32 run as launches over groups of up to 16 rows: the same bar against
    the fp64 product, and each group bit-identical to a separate call on its rows."""
    K, N = 4096, 2048
    w = synthetic_weights(K, N, qtype, seed=31, device=cuda)
    g = torch.Generator(device=cuda).manual_seed(32)
    x = torch.randn(batch, K, generator=g, device=cuda)
    y = vb.gemv_dequant(x, w, None, K, N, qtype)
    ref = x.double() @ vb.dequantize(w, K, N, qtype).double()
    assert ((y.double() - ref).abs().max() / ref.abs().max()).item() <= TOL
    assert torch.equal(y[:16], vb.gemv_dequant(x[:16].contiguous(), w, None, K, N, qtype))
    assert torch.equal(y[16:], vb.gemv_dequant(x[16:].contiguous(), w, None, K, N, qtype))


def test_gemv_1d_x_and_out_buffer(cuda, oracle):
    K, N, t = 256, 768, F.GGML_TYPE_Q4_K
    rng = np.random.default_rng(3)
    w = quantize(rng.normal(0, 0.02, (K, N)).astype(np.float32), t).numpy()
    x = rng.normal(0, 1, K).astype(np.float32)
    out = torch.full((N,), float("nan"), device=cuda)
    res = vb.gemv_dequant(torch.from_numpy(x).to(cuda), torch.from_numpy(w).to(cuda), out, K, N, t,
                          scratch=None)
    assert res.data_ptr() == out.data_ptr()
    assert max_rel(out.cpu().numpy(), oracle.gemv_dequant(x, w, K, N, t)[0]) <= TOL


def test_gemv_zero_k_gives_zeros(cuda):
    w = torch.zeros(0, dtype=torch.uint8, device=cuda)
    x = torch.zeros(0, device=cuda)
    y = vb.gemv_dequant(x, w, torch.full((256,), 7.0, device=cuda), 0, 256, "Q4_K")
    assert torch.count_nonzero(y) == 0


# (K, N) of the BASELINE decode layer (config 2) plus the 70B-shape Q8_0 rows (config 5)
FULL = [(F.GGML_TYPE_Q4_K, 4096, 14336), (F.GGML_TYPE_Q4_K, 14336, 4096),
        (F.GGML_TYPE_Q4_K, 4096, 6144), (F.GGML_TYPE_Q6_K, 4096, 14336),
        (F.GGML_TYPE_Q8_0, 8192, 10240), (F.GGML_TYPE_Q8_0, 28672, 8192)]


@pytest.mark.parametrize("qtype,K,N", FULL)
@pytest.mark.parametrize("batch", [1, 4, 16])
def test_gemv_full_size_vs_fp64(cuda, qtype, K, N, batch):
    w = synthetic_weights(K, N, qtype, seed=0, device=cuda)
    g = torch.Generator(device=cuda).manual_seed(1)
    x = torch.randn(batch, K, generator=g, device=cuda)
    y = vb.gemv_dequant(x, w, None, K, N, qtype)
    deq = vb.dequantize(w, K, N, qtype)  # bit-exact with the reference (tested above)
    ref = x.double() @ deq.double()
    err = ((y.double() - ref).abs().max() / ref.abs().max()).item()
    assert err <= TOL
    # determinism: fixed reduction order -> bitwise repeatable
    y2 = vb.gemv_dequant(x, w, None, K, N, qtype)
    assert torch.equal(y, y2)


@pytest.mark.parametrize("qtype", TYPES)
def test_gemv_linearity_and_row_independence(cuda, qtype):
    K, N = 4096, 4096
    w = synthetic_weights(K, N, qtype, seed=2, device=cuda)
    g = torch.Generator(device=cuda).manual_seed(4)
    x = torch.randn(4, K, generator=g, device=cuda)
    y = vb.gemv_dequant(x, w, None, K, N, qtype)
    y_sum = vb.gemv_dequant((x[0] + x[1]).contiguous(), w, None, K, N, qtype)
    assert ((y_sum - (y[0] + y[1])).abs().max() / y_sum.abs().max()).item() <= TOL
    # each batch row is an independent GEMV: batch 4 row 2 == batch 1 on that row
    y_one = vb.gemv_dequant(x[2].contiguous(), w, None, K, N, qtype)
    # different kernel instantiations (batch 1 vs 4) add in different orders
    assert ((y_one - y[2]).abs().max() / y_one.abs().max()).item() <= 1e-4


@pytest.mark.parametrize("qtype,batch", [(F.GGML_TYPE_Q4_K, 1), (F.GGML_TYPE_Q4_K, 4),
                                         (F.GGML_TYPE_Q8_0, 1), (F.GGML_TYPE_Q6_K, 8)])
def test_gemv_cuda_graph_replay(cuda, qtype, batch):
    """A decode engine captures its GEMVs in a CUDA graph: the captured C-ABI call (cluster
    split-K, or split-K scratch whose counters reset themselves) replays bit-identically to
    the eager call, repeatedly, and follows new contents of the captured x buffer."""
    import ctypes as C
    from vibeblade_b200 import _lib
    lib = _lib.load()
    K, N = 4096, 6144
    w = synthetic_weights(K, N, qtype, seed=21, device=cuda)
    g = torch.Generator(device=cuda).manual_seed(22)
    x = torch.randn(batch, K, generator=g, device=cuda)
    y = torch.empty(batch, N, device=cuda)
    v = C.c_size_t()
    _lib.check(lib.vbq_gemv_scratch_bytes(K, N, qtype, batch, C.byref(v)), lib)
    scratch = torch.zeros(max(int(v.value), 16), dtype=torch.uint8, device=cuda)
    side = torch.cuda.Stream(cuda)

    def call(stream_ptr):
        _lib.check(lib.vbq_gemv(x.data_ptr(), w.data_ptr(), y.data_ptr(), K, N, qtype, batch,
                                scratch.data_ptr(), scratch.numel(), stream_ptr), lib)

    side.wait_stream(torch.cuda.current_stream(cuda))
    with torch.cuda.stream(side):
        call(side.cuda_stream)  # warm-up outside the capture (one-time attribute setup)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            call(side.cuda_stream)
    torch.cuda.current_stream(cuda).wait_stream(side)
    torch.cuda.synchronize()
    for _ in range(2):
        x.copy_(torch.randn(batch, K, generator=g, device=cuda))
        call(torch.cuda.current_stream(cuda).cuda_stream)
        torch.cuda.synchronize()
        y_eager = y.clone()
        y.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(y, y_eager)
    assert vb.device_status() == 0


def _outlier_x(rng, batch, K, frac, lo=100.0, hi=1000.0):
    """N(0, 1) activations with outlier channels, like real hidden states: `frac` of the
    entries of every row scaled by lo..hi (random sign), scattered, so many 32-row warp
    slices hold one outlier among 31 ordinary rows; one extra outlier is placed at the
    last row of the first slice."""
    x = rng.normal(0, 1, (batch, K)).astype(np.float32)
    n = max(1, int(frac * K))
    for b in range(batch):
        idx = rng.choice(K, n, replace=False)
        x[b, idx] *= (rng.uniform(lo, hi, n) * rng.choice([-1.0, 1.0], n)).astype(np.float32)
        x[b, 31] = np.float32(hi)
    return x


def _check_columns(y, ref, what):
    """Max-norm bar (1e-3 of the largest output) and a per-column bar: every output with
    |ref| >= 1e-2 of its row's largest keeps 1e-3 relative accuracy."""
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    mx = np.abs(ref).max(axis=1, keepdims=True)
    err = np.abs(y - ref)
    assert (err / mx).max() <= TOL, f"{what}: max-norm {(err / mx).max():.3g}"
    big = np.abs(ref) >= 1e-2 * mx
    rel = err[big] / np.abs(ref[big])
    assert rel.max() <= TOL, f"{what}: per-column {rel.max():.3g}"


OUTLIER = [(F.GGML_TYPE_Q4_K, 4096, 14336), (F.GGML_TYPE_Q4_K, 14336, 4096),
           (F.GGML_TYPE_Q8_0, 8192, 10240), (F.GGML_TYPE_Q8_0, 28672, 8192),
           (F.GGML_TYPE_Q6_K, 4096, 4096)]


@pytest.mark.parametrize("qtype,K,N", OUTLIER)
@pytest.mark.parametrize("batch", [1, 4, 16])
@pytest.mark.parametrize("frac", [0.001, 0.01])
def test_gemv_outlier_activations(cuda, oracle, qtype, K, N, batch, frac):
    """The integer kernels round x * scale per (warp, batch row) to a fixed point set by
    the slice's largest value, so an outlier coarsens its 31 neighbours: checked per
    column against the fp64 product and against the reference's sequential fp32 sum."""
    rng = np.random.default_rng(K + N + batch + int(frac * 1e4) + qtype)
    w = synthetic_weights(K, N, qtype, seed=K + qtype, device=cuda)
    x = _outlier_x(rng, batch, K, frac)
    y = vb.gemv_dequant(torch.from_numpy(x).to(cuda), w, None, K, N, qtype).cpu().numpy()
    assert vb.device_status() == 0
    deq = vb.dequantize(w, K, N, qtype).double()
    ref64 = (torch.from_numpy(x).to(cuda).double() @ deq).cpu().numpy()
    del deq
    _check_columns(y, ref64, "fp64")
    ref = oracle.gemv_dequant(x, w.cpu().numpy(), K, N, qtype)
    _check_columns(y, ref, "oracle")


# The generic kernel: the MoE router (hidden 4096 -> 8 experts) as GGUF files store it
# (F32 / F16 / BF16), Q8_0 widths that are multiples of 32 but not of 256, and unquantized
# weights of odd widths.
GENERIC = [(F.GGML_TYPE_F32, 4096, 8), (F.GGML_TYPE_F16, 4096, 8), (F.GGML_TYPE_BF16, 4096, 8),
           (F.GGML_TYPE_F32, 6144, 64), (F.GGML_TYPE_F16, 300, 1001), (F.GGML_TYPE_BF16, 2048, 4104),
           (F.GGML_TYPE_Q8_0, 4096, 32), (F.GGML_TYPE_Q8_0, 4096, 1184), (F.GGML_TYPE_Q8_0, 1000, 8288)]


def _weights_of(rng, qtype, K, N):
    vals = rng.normal(0, 0.05, (K, N)).astype(np.float32)
    if qtype == F.GGML_TYPE_F32:
        return vals.view(np.uint8).reshape(K, -1)
    if qtype == F.GGML_TYPE_F16:
        return vals.astype(np.float16).view(np.uint8).reshape(K, -1)
    if qtype == F.GGML_TYPE_BF16:
        return (vals.view(np.uint32) >> 16).astype(np.uint16).view(np.uint8).reshape(K, -1)
    return quantize(vals, qtype).numpy()


@pytest.mark.parametrize("qtype,K,N", GENERIC)
@pytest.mark.parametrize("batch", [1, 3, 4, 16, 32, 37])
def test_gemv_generic_kernel_vs_oracle(cuda, oracle, qtype, K, N, batch):
    rng = np.random.default_rng(K + N + batch + qtype)
    w = _weights_of(rng, qtype, K, N)
    x = rng.normal(0, 1, (batch, K)).astype(np.float32)
    assert vb.gemv_scratch_bytes(K, N, qtype, batch) == 0  # no scratch on this path
    wd = torch.from_numpy(np.ascontiguousarray(w)).to(cuda)
    y = vb.gemv_dequant(torch.from_numpy(x).to(cuda), wd, None, K, N, qtype).cpu().numpy()
    ref = oracle.gemv_dequant(x, w, K, N, qtype)
    _check_columns(y, ref, "oracle")
    y2 = vb.gemv_dequant(torch.from_numpy(x).to(cuda), wd, None, K, N, qtype).cpu().numpy()
    assert np.array_equal(y, y2)  # deterministic (split order fixed)


def test_gemv_router_feeds_moe_routing(cuda, oracle):
    """The reference's MoE router step (cpp/src/fast_model.cpp:861-872) for a prefill's
    tokens in one call: the F32 router GEMV over hidden 4096 -> 8 experts, then softmax and
    top-2; the device routing of the device logits picks the oracle's experts."""
    T, H, E = 300, 4096, 8
    rng = np.random.default_rng(3)
    w = _weights_of(rng, F.GGML_TYPE_F32, H, E)
    x = rng.normal(0, 1, (T, H)).astype(np.float32)
    lg = vb.gemv_dequant(torch.from_numpy(x).to(cuda), torch.from_numpy(w).to(cuda), None, H, E,
                         F.GGML_TYPE_F32)
    ref = oracle.gemv_dequant(x, w, H, E, F.GGML_TYPE_F32)
    _check_columns(lg.cpu().numpy(), ref, "router")
    idx, _ = vb.moe_route(lg, 2)
    idx_ref, _ = vb.moe_route(torch.from_numpy(ref).to(cuda), 2)
    assert torch.equal(idx.sort(dim=1).values, idx_ref.sort(dim=1).values)


@pytest.mark.parametrize("qtype", [F.GGML_TYPE_Q6_K, F.GGML_TYPE_Q4_K, F.GGML_TYPE_Q8_0])
@pytest.mark.parametrize("batch", [1, 4])
def test_gemv_lm_head_vocab_size(cuda, qtype, batch):
    """The lm_head projection at a Llama-3 vocabulary (cpp/src/fast_model.cpp:1022, 1058:
    gemv_dequant_mt over N = vocab): 4096 x 128256 (501 column tiles) in Q6_K, the usual
    type of output.weight in Q4_K_M files, and in Q4_K / Q8_0; against the fp64 product with
    the per-column bar, and bitwise repeatable."""
    K, N = 4096, 128256
    w = synthetic_weights(K, N, qtype, seed=77, device=cuda)
    g = torch.Generator(device=cuda).manual_seed(78)
    x = torch.randn(batch, K, generator=g, device=cuda)
    y = vb.gemv_dequant(x, w, None, K, N, qtype)
    ref = (x.double() @ vb.dequantize(w, K, N, qtype).double()).cpu().numpy()
    _check_columns(y.cpu().numpy(), ref, "fp64")
    assert torch.equal(y, vb.gemv_dequant(x, w, None, K, N, qtype))
    assert vb.device_status() == 0
