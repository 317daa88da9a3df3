"""CPU checks of the MoE restatement against the golden vectors made by the reference's
own vibeblade/moe.py (tests/golden/make_moe_golden.py)."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import load_golden, max_rel
from oracle.moe_oracle import moe_ffn, route, softmax32


def _dense(oracle, g, name, k, n):
    E, t = int(g["E"]), int(g["type"])
    slab = g[name].reshape(E, -1)
    return np.stack([oracle.dequantize(slab[e], k, n, t) for e in range(E)])


def test_route_matches_reference_router():
    g = load_golden("moe_q4_k")
    idx, w = route(g["logits"], int(g["topk"]))
    # the reference's argpartition leaves the order of the k winners unspecified:
    # compare per token as sets, weights matched by expert
    oi, orf = np.argsort(idx, 1), np.argsort(g["idx"], 1)
    assert np.array_equal(np.take_along_axis(idx, oi, 1), np.take_along_axis(g["idx"], orf, 1))
    np.testing.assert_array_equal(np.take_along_axis(w, oi, 1), np.take_along_axis(g["weight"], orf, 1))
    # descending order, rows sum to 1
    assert np.all(np.diff(w, axis=1) <= 0)
    np.testing.assert_allclose(w.sum(1), 1.0, rtol=1e-6)


def test_route_edge_cases():
    # clipping at +-50, exact ties go to the lower index, topk == E
    lg = np.array([[100.0, 50.0, -100.0, 0.0], [1.0, 1.0, 1.0, 1.0], [0.0, 3.0, 3.0, -1.0]],
                  np.float32)
    idx, w = route(lg, 2)
    assert idx[0].tolist() == [0, 1] and np.allclose(w[0], 0.5)  # both clipped to 50
    assert idx[1].tolist() == [0, 1]
    assert idx[2].tolist() == [1, 2]
    idx4, w4 = route(lg, 4)
    np.testing.assert_allclose(w4.sum(1), 1.0, rtol=1e-6)
    np.testing.assert_allclose(softmax32(lg).sum(1), 1.0, rtol=1e-6)


def test_moe_oracle_matches_reference(oracle):
    g = load_golden("moe_q4_k")
    H, I = int(g["H"]), int(g["I"])
    wg, wu, wd = _dense(oracle, g, "gate", H, I), _dense(oracle, g, "up", H, I), _dense(oracle, g, "down", I, H)
    out = moe_ffn(g["x"], g["logits"], wg, wu, wd, int(g["topk"]), "fp32")
    assert max_rel(out, g["out"]) <= 1e-5
    # the bf16-rounding model of the device path stays well inside the GEMM tolerance
    outd = moe_ffn(g["x"], g["logits"], wg, wu, wd, int(g["topk"]), "device")
    assert max_rel(outd, g["out"]) <= 2e-2


def test_moe_oracle_planted_error_is_caught(oracle):
    """A wrong routing weight must move the output by more than the tolerance."""
    g = load_golden("moe_q4_k")
    H, I = int(g["H"]), int(g["I"])
    wg, wu, wd = _dense(oracle, g, "gate", H, I), _dense(oracle, g, "up", H, I), _dense(oracle, g, "down", I, H)
    bad = g["logits"].copy()
    bad[:, 0] += 5.0  # route almost everything to expert 0
    out = moe_ffn(g["x"], bad, wg, wu, wd, int(g["topk"]), "fp32")
    assert max_rel(out, g["out"]) > 2e-2


@pytest.mark.parametrize("T", [0, 1, 5])
def test_moe_oracle_small_batches(oracle, T):
    g = load_golden("moe_q4_k")
    H, I = int(g["H"]), int(g["I"])
    wg, wu, wd = _dense(oracle, g, "gate", H, I), _dense(oracle, g, "up", H, I), _dense(oracle, g, "down", I, H)
    out = moe_ffn(g["x"][:T], g["logits"][:T], wg, wu, wd, int(g["topk"]), "fp32")
    assert out.shape == (T, H)
    if T:
        assert max_rel(out, g["out"][:T]) <= 1e-5
