"""Benchmark of the k-quant dequantize-and-multiply path on B200.

Default workload: one Llama-8B decode layer in Q4_K at batch 1 --
the five projections QKV 4096x6144, o 4096x4096, gate and up 4096x14336, down 14336x4096 --
as fused dequant-GEMVs, in the engine's layout (vibeblade_b200.engine: gate and up packed
into one 4096x28672 matrix, so four launches; the same bytes).  A step is one pass over the
layer.  Weights are synthetic
(N(0, 0.02), seed 0, quantized by vibeblade_b200.quantize); six distinct copies of the
layer rotate so every step streams weights that are not in the 126 MB L2.

Metric: Q4_K dequant-GEMV HBM GB/s = algorithmic bytes (K*N*bpw + B*K*4 + B*N*4 per
GEMV) / device time.  With --gpus N (torchrun), every rank streams its own layer copies
(independent objects, no collective: weak scaling) and the value is the sum over ranks
divided by the max over ranks of the timed region.

--impl reference times the reference's own CPU gemv_dequant (oracle/_ref, compiled from
the reference sources; the C restatement when that library is absent) on the same
workload with all host threads.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "Q4_K dequant-GEMV HBM GB/s"
LAYER_8B = [("qkv", 4096, 6144), ("o", 4096, 4096), ("gate", 4096, 14336), ("up", 4096, 14336),
            ("down", 14336, 4096)]
QTYPE = 12  # Q4_K
BPW = 144 / 256


def layer_bytes(batch: int) -> int:
    return sum(int(K * N * BPW) + batch * K * 4 + batch * N * 4 for _, K, N in LAYER_8B)


def weight_seed(rank: int, copy: int, matrix: int) -> int:
    """Seed of one synthetic weight matrix; both bench arms use these."""
    return 1000 * rank + 10 * copy + matrix


def make_inputs(dev, batch: int, n_copies: int, rank: int):
    """The decode workload's inputs: n_copies distinct copies of the layer's five Q4_K
    matrices (N(0, 0.02) quantized by this library, seeds weight_seed) and x N(0, 1) per
    input width (torch generator seed 1), all on `dev`.  Both bench arms call this, so the
    reference arm times the same bytes the GPU arm streams."""
    import torch
    from vibeblade_b200.quantize import synthetic_weights
    layers = [[(K, N, synthetic_weights(K, N, QTYPE, seed=weight_seed(rank, c, i), device=dev))
               for i, (_, K, N) in enumerate(LAYER_8B)] for c in range(n_copies)]
    g = torch.Generator(device=dev).manual_seed(1)
    xs = {K: torch.randn(batch, K, generator=g, device=dev) for _, K, _ in LAYER_8B}
    return layers, xs


def pack_gate_up(layer):
    """The engine layout of one layer copy (vibeblade_b200.engine.DeviceLayer): gate and up
    side by side in one K x 2N block matrix (each row: gate's blocks, then up's), one launch
    for both; the same bytes as the two matrices."""
    import torch
    (kq, nq, wq), (ko, no, wo), (kg, ng, wg), (_, nu, wu), down = layer
    gu = torch.cat([wg.view(kg, -1), wu.view(kg, -1)], dim=1).contiguous()
    return [(kq, nq, wq), (ko, no, wo), (kg, ng + nu, gu), down]


def bench_config(batch: int, n_copies: int, world: int) -> dict:
    """The workload description both arms print (the same dict in both)."""
    return {"workload": "llama8b_decode_layer_q4k", "batch": batch,
            "matrices": [f"{n} {k}x{m}" for n, k, m in LAYER_8B],
            "gate_up": "the GPU arm runs gate and up as one packed 4096x28672 matrix (the engine "
                       "layout, vibeblade_b200.engine), the reference arm as two gemv_dequant "
                       "calls; the same weight bytes and the same algorithmic bytes per step",
            "weights": "N(0,0.02) quantized Q4_K, seed 1000*rank + 10*copy + matrix; x N(0,1) seed 1",
            "layer_copies_rotated": n_copies,
            "l2": f"inputs larger than L2: {n_copies} distinct layer copies "
                  f"({n_copies * layer_bytes(batch) / 1e6:.0f} MB) rotate per step",
            "parallelism": f"{world} independent GPU(s), own layer copies each (no collective)"}


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", 1400.0)), "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "src": "fallback"}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 20 ms during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "20"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None
        return self

    def __exit__(self, *a):
        if self.p is not None:
            time.sleep(0.25)
            self.p.terminate()
            try:
                self.p.wait(5)
            except subprocess.TimeoutExpired:
                self.p.kill()

    def summary(self) -> dict:
        self.f.flush()
        rows = [r.split(",") for r in Path(self.f.name).read_text().splitlines() if r.strip()]
        os.unlink(self.f.name)
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = max(mx, float(r[2]))
            except (ValueError, IndexError):
                continue
            for n, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(n_gpus: int):
    import torch
    import torch.distributed as dist
    if n_gpus > 1 or int(os.environ.get("WORLD_SIZE", "1")) > 1:
        rank = int(os.environ["RANK"])
        local = int(os.environ.get("LOCAL_RANK", rank))
        torch.cuda.set_device(local)
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        return rank, dist.get_world_size(), local
    return 0, 1, 0


def _time_steps(step, steps: int, warmup: int, stream, world: int):
    """Device time of `steps` calls of step() after `warmup`, max over ranks (ms)."""
    import torch
    import torch.distributed as dist
    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        step(warmup + i)
    e1.record(stream)
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1)], device=torch.device("cuda", torch.cuda.current_device()),
                     dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _soft(fn, *args, **kw) -> dict:
    """A one-GPU extra measurement whose failure is reported on the line instead of ending
    the run (the headline is measured before the extras)."""
    try:
        return fn(*args, **kw)
    except Exception as e:  # noqa: BLE001 - reported on the line, not hidden
        import torch
        torch.cuda.synchronize()
        return {"error": f"{type(e).__name__}: {e}"[:300]}


def _prefill_layer(dev, steps: int, qtype: int, M: int, seed0: int) -> tuple[float, float]:
    """TFLOP/s and ms of the 8B layer's five matrices at M tokens (tcgen05 GEMM, bf16 out):
    qkv, o, then gate and up side by side on two streams (independent GEMMs over the same
    activations, as an engine's FFN and vibeblade_b200.tp run them: 2 x 224 pair tiles at
    M = 2048 fill 7 waves of the 74 SM pairs instead of 2 x 4), then down."""
    import torch
    import vibeblade_b200 as vb
    from vibeblade_b200.quantize import synthetic_weights
    mats = [(K, N, synthetic_weights(K, N, qtype, seed=seed0 + i, device=dev)) for i, (_, K, N) in enumerate(LAYER_8B)]
    g = torch.Generator(device=dev).manual_seed(2)
    acts = {K: torch.randn(M, K, generator=g, device=dev).to(torch.bfloat16) for _, K, _ in LAYER_8B}
    outs = [torch.empty(M, N, device=dev, dtype=torch.bfloat16) for _, _, N in LAYER_8B]
    cur = torch.cuda.current_stream(dev)
    side = torch.cuda.Stream(dev)

    def gemm(i):
        K, N, w = mats[i]
        vb.gemm_dequant(acts[K], w, outs[i], M, K, N, qtype, out_dtype=torch.bfloat16)

    def step(_):
        gemm(0)
        gemm(1)
        side.wait_stream(cur)
        gemm(2)
        with torch.cuda.stream(side):
            gemm(3)
        cur.wait_stream(side)
        gemm(4)

    ms = _time_steps(step, steps, 3, cur, 1)
    flops = sum(2 * M * K * N for _, K, N in LAYER_8B)
    del mats, acts, outs
    torch.cuda.empty_cache()
    return flops * steps / (ms * 1e-3) / 1e12, ms / steps


def bench_prefill(dev, steps: int) -> dict:
    """the 8B layer's five matrices in Q6_K times bf16 activations at
    M = 2048 (the value), 512 and 8192; and the same layer in Q4_K at M = 2048 and 8192 (the
    north star's own GEMM target: Q4_K prefill at >= 55 % of the bf16 peak)."""
    pk, pks = peaks()["bf16_tflops"], peaks()["bf16_tflops_sustained"]
    tf, ms = _prefill_layer(dev, steps, 14, 2048, 200)
    # the steps run back to back for tens of ms under the power cap: both the burst and the
    # sustained cuBLAS figures are given as denominators
    out = {"metric": "Q6_K prefill GEMM TFLOP/s (8B layer, M=2048, bf16 out)", "value": round(tf, 1),
           "unit": "TFLOP/s", "ms_per_layer": round(ms, 4), "steps": steps,
           "frac_of_bf16_peak": round(tf / pk, 4), "frac_of_bf16_sustained": round(tf / pks, 4),
           "kernel": "vbq::gemm::gemm_kernel (2-SM tcgen05, cta_group::2)"}
    for qt, name, Ms in ((14, "q6_k", (512, 8192)), (12, "q4_k", (2048, 8192))):
        for M in Ms:
            t, m = _prefill_layer(dev, max(3, steps // (4 if M == 8192 else 1)), qt, M, 400)
            out[f"{name}_m{M}"] = {"value": round(t, 1), "unit": "TFLOP/s", "ms_per_layer": round(m, 4),
                                   "frac_of_bf16_peak": round(t / pk, 4),
                                   "frac_of_bf16_sustained": round(t / pks, 4)}
    return out


def bench_lm_head(dev, steps: int) -> dict:
    """The lm_head GEMV at a Llama-3 vocabulary (4096 x 128256, batch 1; the reference's
    gemv_dequant_mt at cpp/src/fast_model.cpp:1022) in Q6_K -- the usual type of
    output.weight in Q4_K_M files -- and Q4_K, plus Q6_K at batch 4; two weight copies
    alternate (> L2)."""
    import torch
    import vibeblade_b200 as vb
    from vibeblade_b200.quantize import synthetic_weights
    K, N = 4096, 128256
    out = {"shape": f"{K}x{N}", "batch": 1}
    g = torch.Generator(device=dev).manual_seed(6)
    for t, name, B in ((14, "q6_k", 1), (12, "q4_k", 1), (14, "q6_k_batch4", 4)):
        x = torch.randn(B, K, generator=g, device=dev)
        y = torch.empty(B, N, device=dev)
        ws = [synthetic_weights(K, N, t, seed=300 + i, device=dev) for i in range(2)]
        ms = _time_steps(lambda i: vb.gemv_dequant(x, ws[i % 2], y, K, N, t), 5 * steps, 4,
                         torch.cuda.current_stream(dev), 1)
        nbytes = K * N * (210 if t == 14 else 144) // 256 + 4 * B * (K + N)
        gbs = nbytes * 5 * steps / (ms * 1e-3) / 1e9
        out[name] = {"value": round(gbs, 1), "unit": "GB/s", "us_per_call": round(1e3 * ms / (5 * steps), 2),
                     "frac_of_hbm": round(gbs / peaks()["hbm_gbs"], 4)}
        if B > 1:
            out[name]["batch"] = B
        del ws
    return out


def bench_other_types(dev, steps: int) -> dict:
    """The reference dispatcher's other block types (Q4_0, Q4_1, Q5_0, Q5_1, Q2_K, Q3_K,
    Q5_K, Q8_K) through their staged GEMV kernel: config 2's 4096 x 14336 at batch 1,
    synthetic weights (random codes, N(0, 1e-3) scales); enough copies alternate that they
    never sit in L2 (>= 256 MB)."""
    import torch
    import vibeblade_b200 as vb
    from vibeblade_b200 import formats as F
    from vibeblade_b200.quantize import random_block_weights
    K, N = 4096, 14336
    out = {"shape": f"{K}x{N}", "batch": 1,
           "kernel": ("vbq::gstage::gemv_stage_kernel (per-warp cp.async rings, fp32x2 CUDA-core dot); "
                      "Q5_K: vbq::gmma::gemv_mma_kernel<1, false, true> (the Q4_K u8 x s8 tensor-core "
                      "kernel with the fifth bits merged into its A fragments); Q4_0 / Q4_1 / Q5_0 / "
                      "Q5_1: vbq::gq8::gemv_q8_kernel<1, false, F> (the Q8_0 tensor-core kernel, "
                      "nibbles as u8 codes)")}
    g = torch.Generator(device=dev).manual_seed(8)
    x = torch.randn(1, K, generator=g, device=dev)
    y = torch.empty(1, N, device=dev)
    for t in F.OTHER_BLOCK_TYPES:
        wbytes = K * F.row_bytes(t, N)
        n_copies = max(2, -(-(256 << 20) // wbytes))
        ws = [random_block_weights(K, N, t, seed=500 + i, device=dev) for i in range(n_copies)]
        ms = _time_steps(lambda i: vb.gemv_dequant(x, ws[i % n_copies], y, K, N, t), 5 * steps, 4,
                         torch.cuda.current_stream(dev), 1)
        gbs = (wbytes + 4 * (K + N)) * 5 * steps / (ms * 1e-3) / 1e9
        out[F.TYPE_NAMES[t].lower()] = {"value": round(gbs, 1), "unit": "GB/s",
                                        "us_per_call": round(1e3 * ms / (5 * steps), 2),
                                        "frac_of_hbm": round(gbs / peaks()["hbm_gbs"], 4)}
        del ws
    torch.cuda.empty_cache()
    return out


def bench_moe(dev, steps: int) -> dict:
    """MoE FFN, 8 experts top-2, hidden 4096, intermediate 14336, Q4_K,
    4096 tokens routed by N(0,1) logits (seed 3)."""
    import torch
    import vibeblade_b200 as vb
    from vibeblade_b200.quantize import synthetic_weights
    T, H, I, E, k = 4096, 4096, 14336, 8, 2
    wg = torch.cat([synthetic_weights(H, I, 12, seed=10 + e, device=dev).reshape(-1) for e in range(E)])
    wu = torch.cat([synthetic_weights(H, I, 12, seed=20 + e, device=dev).reshape(-1) for e in range(E)])
    wd = torch.cat([synthetic_weights(I, H, 12, seed=30 + e, device=dev).reshape(-1) for e in range(E)])
    g = torch.Generator(device=dev).manual_seed(3)
    x = torch.randn(T, H, generator=g, device=dev)
    lg = torch.randn(T, E, generator=g, device=dev)
    out = torch.empty(T, H, device=dev)

    def step(_):
        vb.moe_ffn(x, lg, wg, wu, wd, I, 12, topk=k, out=out)

    ms = _time_steps(step, steps, 3, torch.cuda.current_stream(dev), 1)
    tf = 2 * T * k * 3 * H * I * steps / (ms * 1e-3) / 1e12
    return {"metric": "MoE FFN TFLOP/s (8 experts top-2, 4096 tokens, Q4_K)", "value": round(tf, 1),
            "unit": "TFLOP/s", "ms_per_step": round(ms / steps, 3), "steps": steps,
            "frac_of_bf16_peak": round(tf / peaks()["bf16_tflops"], 4),
            "frac_of_bf16_sustained": round(tf / peaks()["bf16_tflops_sustained"], 4)}


def bench_tp(dev, rank: int, world: int, steps: int, prefill: bool = True) -> dict:
    """70B FFN (hidden 8192, intermediate 28672, Q8_0) split over the
    `world` GPUs (gate / up column split, down row split, NCCL all-reduce of the fp32
    output); prefill M = 2048 (whole-job TFLOP/s, the 2-SM GEMM) and decode batch 1 and 16
    (latency, the GEMV).  prefill=False measures the decode side only."""
    import torch
    from vibeblade_b200 import tp
    from vibeblade_b200.quantize import synthetic_weights
    H, I, M = 8192, 28672, 2048
    wg = synthetic_weights(H, I, 8, seed=51, device=dev)
    wu = synthetic_weights(H, I, 8, seed=52, device=dev)
    wd = synthetic_weights(I, H, 8, seed=53, device=dev)
    ffn = tp.TPFFN(wg, wu, wd, H, I, 8, rank, world, dev)
    del wg, wu, wd
    torch.cuda.empty_cache()
    g = torch.Generator(device=dev).manual_seed(2)
    xd = torch.randn(1, H, generator=g, device=dev)
    xd16 = torch.randn(16, H, generator=g, device=dev)
    xd32 = torch.randn(32, H, generator=g, device=dev)
    stream = torch.cuda.current_stream(dev)
    dms = _time_steps(lambda _: ffn.decode(xd), 5 * steps, 5, stream, world)
    dms16 = _time_steps(lambda _: ffn.decode(xd16), 5 * steps, 5, stream, world)
    dms32 = _time_steps(lambda _: ffn.decode(xd32), 5 * steps, 5, stream, world)
    dec = {"decode_b1_us_per_ffn": round(1e3 * dms / (5 * steps), 1),
           "decode_b16_us_per_ffn": round(1e3 * dms16 / (5 * steps), 1),
           "decode_b32_us_per_ffn": round(1e3 * dms32 / (5 * steps), 1)}
    if world > 1:
        # the same decode steps with the down GEMV writing into a buffer the peers map and
        # the one-shot all-reduce over NVLink peer memory (vibeblade_b200.peer) instead
        try:  # set-up fails on every rank together (PeerAllReduce), so all skip alike
            ffn.attach_peer(16, dev)  # batches above 16 keep the collective (TPFFN.attach_peer)
        except RuntimeError as e:
            dec["decode_peer_error"] = str(e)[:200]
        if ffn.peer is not None:
            for b, xb in (("1", xd), ("16", xd16)):
                pms = _time_steps(lambda _: ffn.decode(xb), 5 * steps, 5, stream, world)
                dec[f"decode_b{b}_us_per_ffn_peer"] = round(1e3 * pms / (5 * steps), 1)
            ffn.peer.close()
            ffn.peer = None
    if not prefill:
        return {"metric": "70B FFN decode latency, batch 1 (Q8_0, TP over the job's GPUs)",
                "value": dec["decode_b1_us_per_ffn"], "unit": "us", "higher_is_better": False,
                "tp": world, "scaling": "strong", "steps": 5 * steps, **dec,
                "collective": "torch.distributed all_reduce (NCCL) of the fp32 [B, 8192] decode partial sums; "
                              "*_peer: the one-shot all-reduce over peer memory (vbq_peer_allreduce)"}
    x = torch.randn(M, H, generator=g, device=dev).to(torch.bfloat16)
    ms = _time_steps(lambda _: ffn.prefill(x), steps, 3, stream, world)
    # the same step without the collective (each rank's partial sum only): what the
    # all-reduce adds to the step once its overlap with the second half's GEMMs is counted
    # (at TP = 1 there is no collective and the figures are left out)
    ms_local = _time_steps(lambda _: ffn.prefill(x, reduce=False), steps, 3, stream, world) if world > 1 else ms
    tf = 2 * M * 3 * H * I * steps / (ms * 1e-3) / 1e12
    return {"metric": "70B FFN prefill TFLOP/s (Q8_0, M=2048, TP over the job's GPUs)",
            "value": round(tf, 1), "unit": "TFLOP/s", "tp": world, "scaling": "strong",
            "ms_per_step": round(ms / steps, 4), "steps": steps,
            "ms_per_step_without_collective": round(ms_local / steps, 4) if world > 1 else None,
            "collective_exposed_ms": round((ms - ms_local) / steps, 4) if world > 1 else None, **dec,
            "collective": "torch.distributed all_reduce (NCCL) of the bf16 [M, 8192] prefill partial "
                          "sums (the FFN in two row halves: the first half's all-reduce overlapped "
                          "with the second half's GEMMs) and of the fp32 [B, 8192] decode partial sums; "
                          "decode *_peer: the one-shot all-reduce over peer memory (vbq_peer_allreduce)"}


def _ref_libs():
    """(timed library, its build flags, plain library) of the compiled reference: the AVX2
    release build where the host has AVX2 and FMA, else the plain -O3 build; (None, ...)
    when neither library exists (the C restatement is timed then)."""
    from oracle import load_ref
    from oracle.oracle import load_ref_avx2
    plain = load_ref()
    fast = load_ref_avx2()
    if fast is not None:
        return fast, "-O3 -DNDEBUG -mavx2 -mfma", plain
    return plain, "-O3 -DNDEBUG", plain


def cpu_reference_gbs(layers_np, xs_np, batch: int, seconds: float, threads: int,
                      steps: int | None = None, warmup: int = 0):
    """Time the reference's gemv_dequant over the decode layer on host cores: passes over
    the rotated layer copies `layers_np` ([[(K, N, uint8 array)] per copy]) with inputs
    xs_np ({K: fp32 [batch, K]}), K split across `threads` threads (ctypes releases the
    GIL; the reference's own gemv_dequant_mt ignores its thread count, so this only lets
    the baseline use the host's cores).  Returns (gb_per_s, kind, cores, sample,
    per_step_seconds, flags)."""
    from concurrent.futures import ThreadPoolExecutor
    from oracle import load_oracle

    ref, flags, _ = _ref_libs()
    kind = "reference" if ref is not None else "port"
    pool = ThreadPoolExecutor(threads)
    n_copies = len(layers_np)

    if ref is not None:
        def one_layer(step):
            for K, N, w in layers_np[step % n_copies]:
                ref.gemv_dequant_sliced(xs_np[K], w, K, N, QTYPE, threads, pool)
    else:
        orc = load_oracle()
        threads = 1
        flags = "C restatement (oracle/vbq_oracle.c)"

        def one_layer(step):
            for K, N, w in layers_np[step % n_copies]:
                orc.gemv_dequant(xs_np[K], w, K, N, QTYPE)

    for i in range(warmup):
        one_layer(i)
    times = []
    t_end = time.perf_counter() + seconds
    while (steps is None and (time.perf_counter() < t_end or not times)) or \
            (steps is not None and len(times) < steps):
        t0 = time.perf_counter()
        one_layer(warmup + len(times))
        times.append(time.perf_counter() - t0)
    pool.shutdown()
    total = sum(times)
    gbs = layer_bytes(batch) * len(times) / total / 1e9
    sample = (f"{len(times)} passes over {n_copies} rotated copies of the Llama-8B Q4_K decode layer "
              f"(5 GEMVs, batch {batch}), {total:.1f} s; reference gemv_dequant built with {flags}, "
              f"K split across {threads} threads")
    return gbs, kind, threads, sample, times, flags


def cpu_single_thread(layers_np, xs_np, batch: int, seconds: float) -> dict:
    """The reference's stock path as it runs in its engine: gemv_dequant_mt, which ignores
    its thread count (cpp/src/dequant.cpp:783-792), i.e. one core; the plain -O3 build and,
    where the host supports it, the AVX2 release build."""
    fast, flags, plain = _ref_libs()
    out = {"cores": 1}
    builds = [("O3", plain, "-O3 -DNDEBUG")]
    if fast is not None and fast is not plain:
        builds.append(("avx2", fast, flags))
    for name, lib, fl in builds:
        if lib is None:
            continue
        times = []
        t_end = time.perf_counter() + seconds
        while time.perf_counter() < t_end or not times:
            t0 = time.perf_counter()
            for K, N, w in layers_np[len(times) % len(layers_np)]:
                lib.gemv_dequant(xs_np[K], w, K, N, QTYPE)
            times.append(time.perf_counter() - t0)
        out[name] = {"value": round(layer_bytes(batch) * len(times) / sum(times) / 1e9, 3),
                     "unit": "GB/s", "flags": fl, "passes": len(times)}
    return out


def _host_inputs(batch: int, n_copies: int, rank: int):
    """make_inputs() generated where it is fastest (the GPU when one is visible; the host's
    torch quantizer takes ~10 s per large matrix) and handed over as numpy arrays."""
    import torch
    dev = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")
    if dev.type == "cpu":
        n_copies = 1
    layers, xs = make_inputs(dev, batch, n_copies, rank)
    layers_np = [[(K, N, w.cpu().numpy()) for K, N, w in layer] for layer in layers]
    xs_np = {K: x.cpu().numpy() for K, x in xs.items()}
    return layers_np, xs_np


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    layers_np, xs_np = _host_inputs(args.batch, args.copies, 0)
    gbs, kind, cores, sample, times, flags = cpu_reference_gbs(
        layers_np, xs_np, args.batch, 0.0, threads, steps=args.steps, warmup=args.warmup)
    ms = 1e3 * sum(times) / len(times)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (N(0,0.02) weights quantized Q4_K; x N(0,1))",
        "config": bench_config(args.batch, len(layers_np), args.gpus),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": kind,
                         "sample": sample,
                         "single_thread": cpu_single_thread(layers_np, xs_np, args.batch, 3.0)},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def bench_decode_only(dev, args) -> dict:
    """The headline decode steps alone, launched eagerly through the C ABI (one kernel per
    matrix in stream order): the target of the ncu launch list and captures."""
    import torch
    from vibeblade_b200 import _lib
    lib = _lib.load()
    layers, xs = make_inputs(dev, args.batch, args.copies, 0)
    layers = [pack_gate_up(layer) for layer in layers]
    ys = [torch.empty(args.batch, N, device=dev) for _, N, _ in layers[0]]
    sp = torch.cuda.current_stream(dev).cuda_stream

    def step(s):
        for (K, N, w), y in zip(layers[s % len(layers)], ys):
            _lib.check(lib.vbq_gemv(xs[K].data_ptr(), w.data_ptr(), y.data_ptr(), K, N, QTYPE, args.batch,
                                    None, 0, sp), lib)

    ms = _time_steps(step, args.steps, args.warmup, torch.cuda.current_stream(dev), 1)
    return {"metric": METRIC, "value": round(layer_bytes(args.batch) * args.steps / (ms * 1e-3) / 1e9, 1),
            "unit": "GB/s", "launch": "eager", "steps": args.steps, "launches_per_step": len(ys)}


def run_only(args) -> None:
    """One of the extra measurements on its own (a small, repeatable target for ncu)."""
    import torch
    import torch.distributed as dist
    rank, world, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if args.only == "decode":
        res = bench_decode_only(dev, args)
    elif args.only == "prefill":
        res = bench_prefill(dev, args.extras_steps)
    elif args.only == "moe":
        res = bench_moe(dev, args.extras_steps)
    elif args.only == "lm_head":
        res = bench_lm_head(dev, args.extras_steps)
    elif args.only == "other_types":
        res = bench_other_types(dev, args.extras_steps)
    else:
        res = bench_tp(dev, rank, world, args.extras_steps)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        res.update({"n_gpus": world, "only": args.only})
        print(json.dumps(res), flush=True)


def run_gpu(args) -> None:
    import torch
    import torch.distributed as dist
    import vibeblade_b200 as vb
    from vibeblade_b200 import _lib

    rank, world, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    lib = _lib.load()
    B = args.batch
    n_copies = args.copies
    # weights: n_copies distinct layers (distinct seeds per rank and copy)
    layers, xs = make_inputs(dev, B, n_copies, rank)
    # the CPU baseline reads rank 0's five matrices before they are packed
    layers_np = [[(K, N, w.cpu().numpy()) for K, N, w in layer] for layer in layers] \
        if rank == 0 and not args.no_cpu_baseline else None
    layers = [pack_gate_up(layer) for layer in layers]  # the engine layout: 4 launches per step
    launch_shapes = [(K, N) for K, N, _ in layers[0]]
    torch.cuda.empty_cache()
    g = torch.Generator(device=dev).manual_seed(101)  # other batch sizes' activations
    ys = [torch.empty(B, N, device=dev) for _, N in launch_shapes]
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    need = max(vb.gemv_scratch_bytes(K, N, QTYPE, B) for K, N in launch_shapes)
    scratch = torch.zeros(max(need, 16), dtype=torch.uint8, device=dev)
    sptr, sbytes = scratch.data_ptr(), scratch.numel()

    def launch_layer(c: int, stream_ptr: int):
        for (K, N, w), y in zip(layers[c], ys):
            rc = lib.vbq_gemv(xs[K].data_ptr(), w.data_ptr(), y.data_ptr(), K, N, QTYPE, B,
                              sptr, sbytes, stream_ptr)
            if rc:
                _lib.check(rc, lib)

    for s in range(args.warmup):
        launch_layer(s % n_copies, sp)
    torch.cuda.synchronize()
    # Decode steps are replayed from a CUDA graph, as a decode engine runs them: one graph
    # holds a full rotation of the layer copies (n_copies steps, their 4 GEMV launches chained
    # with programmatic dependent launch, which a graph keeps), and a count of steps that is
    # not a multiple of n_copies ends with eager steps.  --no-graph launches eagerly.
    graph = None
    if not args.no_graph:
        cap = torch.cuda.Stream(dev)
        cap.wait_stream(torch.cuda.current_stream(dev))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=cap):
            for c in range(n_copies):
                launch_layer(c, cap.cuda_stream)
        torch.cuda.current_stream(dev).wait_stream(cap)
        for _ in range(max(1, args.warmup // n_copies)):
            graph.replay()
        torch.cuda.synchronize()

    def run_steps(first: int, count: int):
        """`count` decode steps starting at step index `first` (a multiple of n_copies
        when replayed from the graph)."""
        done = 0
        if graph is not None:
            while count - done >= n_copies:
                graph.replay()  # on the current stream
                done += n_copies
        for s in range(first + done, first + count):
            launch_layer(s % n_copies, sp)

    # ---- timed region: K steps, events on the launching stream ----
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(stream)
        run_steps(0, args.steps)
        e1.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms_total = e0.elapsed_time(e1)
    t = torch.tensor([ms_total], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_total = float(t.item())
    total_bytes = layer_bytes(B) * args.steps * world
    value = total_bytes / (ms_total * 1e-3) / 1e9

    # ---- roofline of the GEMV kernel ----
    # Every launch in the timed region is the GEMV kernel, queued back to back with
    # programmatic dependent launch, so the average launch duration is the timed region
    # divided by the launches and `achieved` equals `value`.  (Per-launch events would
    # serialise the launches and hide the overlap.)  The dominant shape, the packed gate|up
    # 4096x28672, and config 2's 4096x14336 alone are also timed on their own.
    achieved = value / world

    def time_shape(mats, K, N):
        yy = torch.empty(B, N, device=dev)
        for i in range(3):
            lib.vbq_gemv(xs[K].data_ptr(), mats[i % len(mats)].data_ptr(), yy.data_ptr(), K, N, QTYPE, B,
                         sptr, sbytes, sp)
        e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        nrep = max(1, args.steps)
        e2.record(stream)
        for i in range(nrep):
            lib.vbq_gemv(xs[K].data_ptr(), mats[i % len(mats)].data_ptr(), yy.data_ptr(), K, N, QTYPE, B,
                         sptr, sbytes, sp)
        e3.record(stream)
        torch.cuda.synchronize()
        nbytes = int(K * N * BPW) + B * (K + N) * 4
        return nbytes * nrep / (e2.elapsed_time(e3) * 1e-3) / 1e9

    gu_gbs = time_shape([layer[2][2] for layer in layers], 4096, 28672)
    from vibeblade_b200.quantize import synthetic_weights
    sep = [synthetic_weights(4096, 14336, QTYPE, seed=900 + i, device=dev) for i in range(4)]
    big_gbs = time_shape(sep, 4096, 14336)
    del sep
    traffic = None
    tp = ROOT / "profiles" / "gemv_q4k_decode_layer_engine_b1.txt"
    if tp.exists():  # dram bytes per launch from the committed ncu capture of this shape
        for line in tp.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch:"):
                traffic = int(line.split(":")[1].strip())

    # ---- end to end through the public API with host buffers ----
    # A step's inputs (x of the 4096-row and 14336-row matrices) sit back to back in one
    # pinned host buffer and one device buffer, its four outputs likewise: one host-to-device
    # copy, four gemv_dequant calls (gate|up packed) writing into views of the output buffer, one
    # device-to-host copy.
    in_ks = sorted(xs)
    x_sizes = [B * K for K in in_ks]
    y_sizes = [B * N for _, N in launch_shapes]
    xh_all = torch.cat([xs[K].reshape(-1).cpu() for K in in_ks]).pin_memory()
    yh_all = torch.empty(sum(y_sizes), pin_memory=True)
    xd_all = torch.empty(sum(x_sizes), device=dev)
    yd_all = torch.empty(sum(y_sizes), device=dev)
    xd = {K: v.view(B, K) for K, v in zip(in_ks, torch.split(xd_all, x_sizes))}
    yd = [v.view(B, N) for (_, N), v in zip(launch_shapes, torch.split(yd_all, y_sizes))]
    h2d = xh_all.numel() * 4
    d2h = yh_all.numel() * 4

    def e2e_step(s: int):
        xd_all.copy_(xh_all, non_blocking=True)
        for (K, N, w), yo in zip(layers[s % n_copies], yd):
            vb.gemv_dequant(xd[K], w, yo, K, N, QTYPE)
        yh_all.copy_(yd_all, non_blocking=True)

    def timed_steps(step_fn, extra_streams=()) -> float:
        for s in range(args.warmup):
            step_fn(s)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for x_s in extra_streams:
            x_s.wait_stream(stream)
        for s in range(args.steps):
            step_fn(s)
        for x_s in extra_streams:
            stream.wait_stream(x_s)
        b.record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([a.elapsed_time(b)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return layer_bytes(B) * args.steps * world / (float(t.item()) * 1e-3) / 1e9

    # every copy in the stream between the GEMVs: the launches cannot overlap a copy
    e2e_serial_value = timed_steps(e2e_step)

    # The same work pipelined, as a serving loop runs it: two slots of pinned host and device
    # buffers; step s's copies run on a copy stream (ordered by events) and overlap the
    # GEMVs of steps s - 1 and s + 1 on the compute stream.  Every step still copies its
    # inputs in and its outputs out inside the timed region.
    copy_st = torch.cuda.Stream(dev)
    slots = []
    for _ in range(2):
        xh_s = xh_all.clone().pin_memory()
        yh_s = torch.empty(sum(y_sizes), pin_memory=True)
        xd_s = torch.empty(sum(x_sizes), device=dev)
        yd_s = torch.empty(sum(y_sizes), device=dev)
        slots.append({"xh": xh_s, "yh": yh_s, "xd_all": xd_s, "yd_all": yd_s,
                      "xd": {K: v.view(B, K) for K, v in zip(in_ks, torch.split(xd_s, x_sizes))},
                      "yd": [v.view(B, N) for (_, N), v in zip(launch_shapes, torch.split(yd_s, y_sizes))],
                      "h2d": torch.cuda.Event(), "gemv": torch.cuda.Event(), "d2h": torch.cuda.Event()})

    def issue_h2d(s: int):
        sl = slots[s % 2]
        copy_st.wait_event(sl["gemv"])  # step s - 2's GEMVs are done with this slot's x
        with torch.cuda.stream(copy_st):
            sl["xd_all"].copy_(sl["xh"], non_blocking=True)
        sl["h2d"].record(copy_st)

    def e2e_pipelined_step(s: int):
        # step s's input copy was issued one step ahead (the first by the timed region's
        # first call); issue step s + 1's now, so that it runs under this step's GEMVs
        if s == 0:
            issue_h2d(0)
        issue_h2d(s + 1)
        sl = slots[s % 2]
        stream.wait_event(sl["h2d"])
        stream.wait_event(sl["d2h"])    # step s - 2's read of this slot's y is done
        for (K, N, w), yo in zip(layers[s % n_copies], sl["yd"]):
            vb.gemv_dequant(sl["xd"][K], w, yo, K, N, QTYPE)
        sl["gemv"].record(stream)
        copy_st.wait_event(sl["gemv"])
        with torch.cuda.stream(copy_st):
            sl["yh"].copy_(sl["yd_all"], non_blocking=True)
        sl["d2h"].record(copy_st)

    e2e_value = timed_steps(e2e_pipelined_step, (copy_st,))

    # the same step (one copy in, four gemv_dequant calls, one copy out) captured once per
    # rotation of the layer copies in a CUDA graph and replayed, as a decode engine runs its
    # step: the copies still happen every step, the per-call host work does not
    e2e_graph_value = None
    if not args.no_graph:
        cap_e = torch.cuda.Stream(dev)
        cap_e.wait_stream(stream)
        graph_e = torch.cuda.CUDAGraph()
        with torch.cuda.stream(cap_e):
            with torch.cuda.graph(graph_e, stream=cap_e):
                for c in range(n_copies):
                    e2e_step(c)
        stream.wait_stream(cap_e)
        graph_e.replay()
        torch.cuda.synchronize()
        reps = max(1, args.steps // n_copies)
        a_g, b_g = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a_g.record(stream)
        for _ in range(reps):
            graph_e.replay()
        b_g.record(stream)
        torch.cuda.synchronize()
        t_g = torch.tensor([a_g.elapsed_time(b_g)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t_g, op=dist.ReduceOp.MAX)
        e2e_graph_value = layer_bytes(B) * reps * n_copies * world / (float(t_g.item()) * 1e-3) / 1e9
        del graph_e

    # The pipelined schedule itself captured in a CUDA graph: per rotation of R steps, the
    # two slots, the copy stream and the events become graph dependencies, so each step's
    # copies overlap the neighbouring steps' GEMVs with no host work per call.  Every step
    # still copies its inputs in from pinned host memory and its outputs out.  Replays run
    # one after another on the stream, so each replay starts with both slots free.
    e2e_graph_pipelined_value = None
    if not args.no_graph:
        R = n_copies if n_copies % 2 == 0 else 2 * n_copies
        cap_p, copy_p = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        cap_p.wait_stream(stream)
        graph_p = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph_p, stream=cap_p):
            copy_p.wait_stream(cap_p)  # fork the copy stream into the capture
            ev = [{"h2d": torch.cuda.Event(), "gemv": torch.cuda.Event(), "d2h": torch.cuda.Event()}
                  for _ in range(2)]

            def g_h2d(s: int):
                sl, e = slots[s % 2], ev[s % 2]
                if s >= 2:
                    copy_p.wait_event(e["gemv"])  # step s - 2's GEMVs are done with this slot's x
                with torch.cuda.stream(copy_p):
                    sl["xd_all"].copy_(sl["xh"], non_blocking=True)
                e["h2d"].record(copy_p)

            g_h2d(0)
            for s in range(R):
                if s + 1 < R:
                    g_h2d(s + 1)
                sl, e = slots[s % 2], ev[s % 2]
                cap_p.wait_event(e["h2d"])
                if s >= 2:
                    cap_p.wait_event(e["d2h"])  # step s - 2's read of this slot's y is done
                with torch.cuda.stream(cap_p):
                    for (K, N, w), yo in zip(layers[s % n_copies], sl["yd"]):
                        vb.gemv_dequant(sl["xd"][K], w, yo, K, N, QTYPE)
                e["gemv"].record(cap_p)
                copy_p.wait_event(e["gemv"])
                with torch.cuda.stream(copy_p):
                    sl["yh"].copy_(sl["yd_all"], non_blocking=True)
                e["d2h"].record(copy_p)
            cap_p.wait_stream(copy_p)  # join
        stream.wait_stream(cap_p)
        graph_p.replay()
        torch.cuda.synchronize()
        reps = max(1, args.steps // R)
        a_p, b_p = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a_p.record(stream)
        for _ in range(reps):
            graph_p.replay()
        b_p.record(stream)
        torch.cuda.synchronize()
        t_p = torch.tensor([a_p.elapsed_time(b_p)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t_p, op=dist.ReduceOp.MAX)
        e2e_graph_pipelined_value = layer_bytes(B) * reps * R * world / (float(t_p.item()) * 1e-3) / 1e9
        del graph_p

    # ---- config 2's other batch sizes: the same rotated layers at batch 4 and 16 ----
    decode_batches = {}
    if B == 1 and not args.no_extras:
        for bx in (4, 16):
            xb = {K: torch.randn(bx, K, generator=g, device=dev) for _, K, _ in LAYER_8B}
            yb = [torch.empty(bx, N, device=dev) for _, N in launch_shapes]
            need_b = max(vb.gemv_scratch_bytes(K, N, QTYPE, bx) for K, N in launch_shapes)
            scr_b = torch.zeros(max(need_b, 16), dtype=torch.uint8, device=dev)

            def layer_b(c: int, stream_ptr: int):
                for (K, N, w), y in zip(layers[c], yb):
                    rc = lib.vbq_gemv(xb[K].data_ptr(), w.data_ptr(), y.data_ptr(), K, N, QTYPE, bx,
                                      scr_b.data_ptr(), scr_b.numel(), stream_ptr)
                    if rc:
                        _lib.check(rc, lib)

            cap_b = torch.cuda.Stream(dev)
            cap_b.wait_stream(stream)
            with torch.cuda.stream(cap_b):
                for c in range(n_copies):
                    layer_b(c, cap_b.cuda_stream)
                graph_b = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph_b, stream=cap_b):
                    for c in range(n_copies):
                        layer_b(c, cap_b.cuda_stream)
            stream.wait_stream(cap_b)
            graph_b.replay()
            torch.cuda.synchronize()
            reps = max(1, args.steps // n_copies)
            a_b, b_b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a_b.record(stream)
            for _ in range(reps):
                graph_b.replay()
            b_b.record(stream)
            torch.cuda.synchronize()
            t_b = torch.tensor([a_b.elapsed_time(b_b)], device=dev, dtype=torch.float64)
            if world > 1:
                dist.all_reduce(t_b, op=dist.ReduceOp.MAX)
            ms_b = float(t_b.item())
            gbs_b = layer_bytes(bx) * reps * n_copies * world / (ms_b * 1e-3) / 1e9
            decode_batches[str(bx)] = {"value": round(gbs_b, 1), "unit": "GB/s",
                                       "us_per_step": round(1e3 * ms_b / (reps * n_copies), 2),
                                       "frac_of_hbm": round(gbs_b / world / peaks()["hbm_gbs"], 4)}
            del graph_b

    # ---- configs 3-5: prefill GEMM, MoE (one GPU) and the tensor-parallel 70B FFN ----
    extras = {}
    if not args.no_extras:
        if world == 1:
            extras["prefill"] = _soft(bench_prefill, dev, args.extras_steps)
            extras["moe"] = _soft(bench_moe, dev, args.extras_steps)
            extras["lm_head"] = _soft(bench_lm_head, dev, args.extras_steps)
            extras["other_types"] = _soft(bench_other_types, dev, args.extras_steps)
        extras["tp_ffn"] = bench_tp(dev, rank, world, args.extras_steps)
    else:  # config 5's decode side runs on the GEMV alone
        extras["tp_ffn_decode"] = bench_tp(dev, rank, world, args.extras_steps, prefill=False)

    pk = peaks()
    line = None
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_total / args.steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (N(0,0.02) weights quantized Q4_K; x N(0,1))",
            "config": bench_config(B, n_copies, world),
            "launch": (f"CUDA graph of {n_copies} steps ({4 * n_copies} GEMV kernels chained by "
                       "programmatic dependent launch), replayed; remainder eager"
                       if graph is not None else "eager, one C-ABI call per GEMV"),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"],
                         "unit": "GB/s", "frac": round(achieved / pk["hbm_gbs"], 4),
                         "traffic": traffic, "traffic_launch": "packed gate|up 4096x28672 (ncu, read + write)",
                         "peak_src": pk["src"] + " (MEASURED_PEAKS.json hbm_gbs)",
                         "kernel": (f"vbq::gmma::gemv_mma_kernel<{1 if B == 1 else 2 if B == 2 else 4}> "
                                    "(u8 x s8 mma.sync, split-K in a thread-block cluster)" if B <= 4
                                    else f"vbq::gwide::gemv_wide_kernel<{8 if B <= 8 else 16}> "
                                    "(u8 x s8 mma.sync, B table shared by warp pairs)"),
                         "gemv_4096x14336_gbs": round(big_gbs, 1),
                         "gemv_4096x14336_frac": round(big_gbs / pk["hbm_gbs"], 4),
                         "gemv_gate_up_4096x28672_gbs": round(gu_gbs, 1),
                         "gemv_gate_up_4096x28672_frac": round(gu_gbs / pk["hbm_gbs"], 4)},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "api": "vibeblade_b200.gemv_dequant",
                    "schedule": ("pinned host buffers, two slots; each step's host-to-device copy "
                                 "issued one step ahead and its device-to-host copy after its "
                                 "gemv_dequant calls, both on a copy stream overlapping the "
                                 "neighbouring steps' GEMVs (one extra input copy per timed run)"),
                    "serial_value": round(e2e_serial_value, 2),
                    "graph_replayed_value": (round(e2e_graph_value, 2)
                                             if e2e_graph_value is not None else None),
                    "graph_pipelined_value": (round(e2e_graph_pipelined_value, 2)
                                              if e2e_graph_pipelined_value is not None else None),
                    "graph_note": ("graph_replayed_value: the serial step (copy in, four calls, "
                                   "copy out) captured and replayed; graph_pipelined_value: the "
                                   "pipelined schedule above captured per rotation of steps and "
                                   "replayed, copies every step; value stays the eager schedule, "
                                   "which calls the API on every step")},
            "gpu_launches": args.steps * len(launch_shapes),
            "clocks": clk.summary(),
        }
        if decode_batches:  # outside the timed region above; same layers, graph-replayed
            line["decode_layer_by_batch"] = decode_batches
        line.update(extras)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        if not args.no_cpu_baseline:
            # the same bytes the GPU streamed (rank 0's copies, as five matrices), rotated alike
            xs_np = {K: x.cpu().numpy() for K, x in xs.items()}
            gbs, kind, cores, sample, _, _ = cpu_reference_gbs(layers_np, xs_np, B, args.cpu_seconds,
                                                               os.cpu_count() or 1)
            line["cpu_baseline"] = {"value": round(gbs, 3), "unit": "GB/s", "cores": cores,
                                    "kind": kind, "sample": sample,
                                    "single_thread": cpu_single_thread(layers_np, xs_np, B, 3.0)}
        print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--copies", type=int, default=6)
    ap.add_argument("--impl", default="vbq", choices=["vbq", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true",
                    help="launch the decode step's GEMVs eagerly instead of replaying a CUDA graph")
    ap.add_argument("--extras", action="store_true",
                    help="(default) also measure the prefill GEMM, MoE and tensor-parallel FFN")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip those; config 5 is then measured on its decode side only")
    ap.add_argument("--extras-steps", type=int, default=10)
    ap.add_argument("--only", choices=["decode", "prefill", "moe", "lm_head", "other_types", "tp"],
                    help="run just this measurement and print its JSON object")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.only:
        run_only(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
