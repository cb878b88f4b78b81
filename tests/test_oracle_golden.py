"""Pin the CPU oracle against the reference's own elementwise expression table
(golden: tests/golden/elementwise_ops.json, generated from the reference source by
tests/golden/make_golden.py). Every op, every edge-case input pair, bit for bit
(NaN payloads compared as NaN) — except ``tanh``, which is checked in the oracle's
"reference" mode (the reference's formula) — plus the device expression table's
op set and arity against the reference's."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from metellus_b200.compute import elementwise as ew
from oracle import ir_eval

G = json.loads((Path(__file__).parent / "golden" / "elementwise_ops.json").read_text())


def _f32(hexes):
    return np.array([int(h, 16) for h in hexes], dtype=np.uint32).view(np.float32)


XS = _f32(G["inputs_hex"])
N = len(XS)
X2 = np.repeat(XS, N)
Y2 = np.tile(XS, N)
C2 = _f32(G["cond_hex"])


def test_op_set_matches_reference():
    assert set(G["ops"]) == set(ew.supported_elementwise_ops())
    for op, d in G["ops"].items():
        assert ew.elementwise_arity(op) == d["arity"]


@pytest.mark.parametrize("op", sorted(G["ops"]))
def test_oracle_matches_reference_table(op):
    d = G["ops"][op]
    want = _f32(d["out_hex"])
    if d["arity"] == 1:
        got = ir_eval.unary(op, XS.copy(), tanh_mode="reference")
    elif d["arity"] == 2:
        got = ir_eval.binary(op, X2.copy(), Y2.copy())
    else:
        got = ir_eval.ternary(op, X2.copy(), Y2.copy(), C2.copy())
    got = np.asarray(got, np.float32)
    both_nan = np.isnan(got) & np.isnan(want)
    same = (got.view(np.uint32) == want.view(np.uint32)) | both_nan
    assert same.all(), f"{op}: {int((~same).sum())} mismatches, first at {np.argmax(~same)}: " \
                       f"got {got[~same][:3]} want {want[~same][:3]}"


def test_tanh_exact_mode_close_to_reference_formula():
    """The device uses CUDA tanhf; the oracle's exact mode (np.tanh) and the
    reference formula agree to fp32 rounding away from 0, where the formula cancels."""
    x = np.linspace(-20, 20, 4001, dtype=np.float32)
    x = x[np.abs(x) > 0.5]
    a = ir_eval.unary("tanh", x, "exact")
    b = ir_eval.unary("tanh", x, "reference")
    np.testing.assert_allclose(a, b, rtol=3e-7, atol=0)
