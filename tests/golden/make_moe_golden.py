"""Generate tests/golden/moe_q4_k.npz from the reference's own MoE code.

Run where the reference checkout is mounted ($VB_REF names it; oracle/build.py holds
the default):

    python tests/golden/make_moe_golden.py

Sources of truth:
* expert weights: this library's Q4_K quantizer output, dequantized by the reference's
  ``vibeblade::dequantize_row`` (cpp/src/dequant.cpp:268-301) compiled into
  oracle/_ref/libvbref.so;
* routing and the expert FFN: ``ExpertRouter.route`` and ``moe_ffn_silu`` of the
  reference's vibeblade/moe.py (:170-206, :407-505), imported by file path.  The router
  is given an identity weight so that ``route`` sees the fixture's logits; the expert
  computation receives the tokens' hidden states.

Slabs are stored in the library's layout: E K x N matrices in the reference block layout,
back to back (gate / up: K = H, N = I; down: K = I, N = H).
"""
from __future__ import annotations

import importlib.util
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.dont_write_bytecode = True  # never write into the read-only reference checkout

from oracle.build import ref_root  # noqa: E402
from oracle.oracle import load_ref  # noqa: E402
from vibeblade_b200 import formats as F  # noqa: E402
from vibeblade_b200.quantize import quantize  # noqa: E402

REF = ref_root()
T, H, I, E, TOPK = 48, 256, 512, 4, 2
QT = F.GGML_TYPE_Q4_K


def _ref_moe():
    spec = importlib.util.spec_from_file_location("_vb_ref_moe", REF / "vibeblade" / "moe.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod  # its dataclasses look the module up by name
    spec.loader.exec_module(mod)
    return mod


class _FixedRouter:
    """Hands moe_ffn_silu the reference router's decision for the fixture's logits."""

    def __init__(self, router, logits):
        self.topk = router.topk
        self._decision = router.route(logits)

    def route(self, x):
        return self._decision


def main() -> None:
    ref = load_ref()
    if ref is None:
        raise SystemExit("reference sources not found; set VB_REF")
    moe = _ref_moe()
    rng = np.random.default_rng(4)
    slabs, dense = {}, {}
    for name, k, n in (("gate", H, I), ("up", H, I), ("down", I, H)):
        qs, ds = [], []
        for e in range(E):
            w = rng.normal(0.0, 0.02, size=(k, n)).astype(np.float32)
            q = quantize(w, QT).numpy()
            qs.append(q.reshape(-1))
            ds.append(np.stack([ref.dequantize_row(q[r], n, QT) for r in range(k)]))
        slabs[name] = np.concatenate(qs)
        dense[name] = np.stack(ds)  # [E, k, n]
    x = np.random.default_rng(1).normal(0.0, 1.0, size=(T, H)).astype(np.float32)
    logits = np.random.default_rng(3).normal(0.0, 1.0, size=(T, E)).astype(np.float32)
    router = moe.ExpertRouter(np.eye(E, dtype=np.float32), TOPK)
    idx, wts = router.route(logits)
    # MoEExpertSet holds gate/up as [E, I, H] and down as [E, H, I] (GGUF order) and
    # transposes them back for its einsums
    experts = moe.MoEExpertSet(dense["gate"].transpose(0, 2, 1), dense["up"].transpose(0, 2, 1),
                               dense["down"].transpose(0, 2, 1))
    out, _ = moe.moe_ffn_silu(x, _FixedRouter(router, logits), experts)
    np.savez_compressed(
        HERE / "moe_q4_k.npz", gate=slabs["gate"], up=slabs["up"], down=slabs["down"],
        x=x, logits=logits,
        idx=np.asarray(idx, np.int32), weight=np.asarray(wts, np.float32),
        out=np.asarray(out, np.float32), T=T, H=H, I=I, E=E, topk=TOPK, type=QT)
    print("moe_q4_k.npz", out.shape, float(np.abs(out).max()))


if __name__ == "__main__":
    main()
