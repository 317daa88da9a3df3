"""Generate tests/golden/layer_llama.npz from the reference's own transformer block.

Run where the reference checkout is mounted ($VB_REF names it; oracle/build.py holds the
default):

    python tests/golden/make_layer_golden.py

Source of truth: ``forward_token`` of the reference's Python engine
(vibeblade/transformer.py:232-325: RMSNorm, Q/K/V, RoPE, grouped-query attention over the
KV cache, o projection + residual, RMSNorm, SwiGLU FFN + residual), imported by path and
run on four positions in turn.  Its weights are the quantized matrices of this fixture
dequantized by the oracle (oracle/vbq_oracle.c: bit-exact with the reference's C++
dequantize_row for Q4_K / Q6_K, and with the GGUF fp16-scale Q8_0 block of the reference's
CUDA kernel and numpy loader, not its C++ reader's float32-scale defect), transposed into
the (out, in) orientation forward_token multiplies by.  The fixture keeps the raw quantized
bytes, so the device engine reads exactly the weights the reference used.
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.dont_write_bytecode = True  # never write into the read-only reference checkout

from oracle.build import ref_root  # noqa: E402
from oracle import load_oracle  # noqa: E402
from oracle.oracle import load_ref  # noqa: E402
from vibeblade_b200 import formats as F  # noqa: E402
from vibeblade_b200.quantize import quantize  # noqa: E402

REF = ref_root()
HIDDEN, N_HEADS, N_KV, FFN, EPS, POSITIONS = 512, 8, 4, 1024, 1e-5, 4
HEAD_DIM = HIDDEN // N_HEADS
# (name, K rows = input width, N columns = output width, type): every quantized type of the
# path; attn_v and ffn_down in Q6_K as Q4_K_M files keep them
MATS = [("attn_q", HIDDEN, HIDDEN, F.GGML_TYPE_Q4_K), ("attn_k", HIDDEN, N_KV * HEAD_DIM, F.GGML_TYPE_Q4_K),
        ("attn_v", HIDDEN, N_KV * HEAD_DIM, F.GGML_TYPE_Q6_K), ("attn_output", HIDDEN, HIDDEN, F.GGML_TYPE_Q8_0),
        ("ffn_gate", HIDDEN, FFN, F.GGML_TYPE_Q4_K), ("ffn_up", HIDDEN, FFN, F.GGML_TYPE_Q4_K),
        ("ffn_down", FFN, HIDDEN, F.GGML_TYPE_Q6_K)]


def _ref_transformer():
    spec = importlib.util.spec_from_file_location("_vb_ref_transformer", REF / "vibeblade" / "transformer.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    return mod


def main() -> None:
    ref = load_ref()
    if ref is None or not (REF / "vibeblade" / "transformer.py").exists():
        raise SystemExit("reference sources not found; set VB_REF")
    tr = _ref_transformer()
    orc = load_oracle()
    rng = np.random.default_rng(2024)
    out = {"hidden": HIDDEN, "n_heads": N_HEADS, "n_kv_heads": N_KV, "ffn": FFN, "eps": EPS}
    weights = {}
    for name, K, N, t in MATS:
        w = quantize(rng.normal(0, 0.05, (K, N)).astype(np.float32), t).numpy()
        deq = orc.dequantize(w, K, N, t)  # [K, N]
        if t != F.GGML_TYPE_Q8_0:  # the pin: identical to the compiled reference
            assert np.array_equal(deq.view(np.uint32),
                                  np.stack([ref.dequantize_row(w[k], N, t) for k in range(K)]).view(np.uint32))
        weights[f"blk.0.{name}.weight"] = deq.T.copy()  # (out, in), as forward_token multiplies
        out[f"{name}_bytes"] = w
        out[f"{name}_type"] = t
    for name in ("attn_norm", "ffn_norm"):
        v = (1.0 + 0.1 * rng.normal(0, 1, HIDDEN)).astype(np.float32)
        weights[f"blk.0.{name}.weight"] = v
        out[name] = v
    x = rng.normal(0, 1, (POSITIONS, HIDDEN)).astype(np.float32)
    cos, sin = tr.build_rope_cache(HEAD_DIM, 64)
    kc = vc = None
    ys = []
    for pos in range(POSITIONS):
        y, kc, vc = tr.forward_token(x[pos:pos + 1], weights, 0, cos, sin, kc, vc, position=pos,
                                     n_heads=N_HEADS, n_kv_heads=N_KV, eps=EPS)
        ys.append(y[0].astype(np.float32))
    out["x"] = x
    out["y"] = np.stack(ys)
    np.savez_compressed(HERE / "layer_llama.npz", **out)
    print("wrote", HERE / "layer_llama.npz")


if __name__ == "__main__":
    main()
