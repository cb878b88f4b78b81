"""GPU parity at the benchmark configurations' FULL shapes.

Each program runs once at its full size through the public ``run`` API on the B200.
Rows (C2, C3, C5) and heads (C4) are independent in these programs, so the oracle
checks sampled rows / heads — the first and last blocks (the last wave of CTAs and the
ragged tail of the grid), a middle block and scattered random rows — by evaluating the
same program on just those rows in fp64 (ground truth) and fp32 (the reference
semantics). C1 and the whole-tensor sum are checked whole. Tolerances: tests/tolerances.py
(the matmul bound 1e-5 normwise is the one BASELINE's matmul programs state; the
reference's own matmul checks are looser, 1e-3 / 1e-2 at bench_matmul.py:189).
"""

from __future__ import annotations

import numpy as np
import pytest

from metellus_b200 import configs, run
from oracle.ir_eval import evaluate
from tests.tolerances import assert_elementwise_close, assert_matmul_close

pytestmark = pytest.mark.gpu


def _rows(n: int, block: int = 64, scattered: int = 64, seed: int = 0) -> np.ndarray:
    r = np.random.default_rng(seed)
    parts = [np.arange(0, block), np.arange(n // 2 - block // 2, n // 2 + block // 2),
             np.arange(n - block, n), r.choice(n, scattered, replace=False)]
    return np.unique(np.concatenate(parts))


def test_c1_full(cuda_device):
    c = configs.CONFIGS["c1"]
    ops = c.build(**c.full)
    res = run(ops)
    assert len(res.groups) == 1
    r64, r32 = evaluate(ops, np.float64), evaluate(ops, np.float32)
    assert_matmul_close(res.env["C"], r64["C"], r32["C"], what="C1 full")


def test_c2_full(cuda_device):
    c = configs.CONFIGS["c2"]
    ops = c.build(**c.full)
    res = run(ops)
    assert len(res.groups) == 1
    out = res.env["out"]
    assert out.shape == (8192, 8192)
    rows = _rows(8192)
    u = ops.uploads
    sub = configs.elementwise_dag_ops(u["x"][rows], u["y"][rows], u["z"][rows])
    r64 = evaluate(sub, np.float64)
    assert_elementwise_close(out[rows], r64["out"], abs_=5e-7, what="C2 full, sampled rows")
    assert np.isfinite(out).all()


def test_c3_full(cuda_device):
    c = configs.CONFIGS["c3"]
    ops = c.build(**c.full)
    res = run(ops)
    assert len(res.groups) == 1
    probs = res.env["probs"]
    rows = _rows(32768, seed=1)
    sub = configs.row_softmax(X=ops.uploads["X"][rows])
    r64 = evaluate(sub, np.float64)
    assert_elementwise_close(probs[rows], r64["probs"], rel=2e-6, abs_=1e-9, what="C3 full, sampled rows")
    # size-independent property over the whole grid: every row sums to 1
    s = probs.astype(np.float64).sum(axis=1)
    assert np.abs(s - 1.0).max() < 1e-4


def test_c3sum_full(cuda_device):
    c = configs.CONFIGS["c3sum"]
    ops = c.build(**c.full)
    res = run(ops)
    X = ops.uploads["X"]
    ref = float(X.astype(np.float64).sum())
    scale = float(np.abs(X).astype(np.float64).sum())
    got = float(res.env["total"][0])
    assert abs(got - ref) <= 1e-6 * scale, (got, ref, scale)


def test_c4_full(cuda_device):
    c = configs.CONFIGS["c4"]
    ops = c.build(**c.full)
    res = run(ops)
    assert len(res.groups) == 1
    O = res.env["O"]
    u = ops.uploads
    for h in (0, 37, 90, 127):
        sub = configs.attention_ops(u["Q"][h:h + 1], u["K"][h:h + 1], u["V"][h:h + 1])
        r64, r32 = evaluate(sub, np.float64), evaluate(sub, np.float32)
        assert_matmul_close(O[h:h + 1], r64["O"], r32["O"], what=f"C4 full, head {h}")


def test_c5_full(cuda_device):
    """Includes the K = 8192 down-projection (U @ W2) at its full size."""
    c = configs.CONFIGS["c5"]
    ops = c.build(**c.full)
    res = run(ops)
    out = res.env["out"]
    rows = _rows(16384, block=32, scattered=32, seed=2)
    u = ops.uploads
    sub = configs.mlp_ops(u["X"][rows], u["W1"], u["W3"], u["W2"], u["b1"], u["b2"])
    r64, r32 = evaluate(sub, np.float64), evaluate(sub, np.float32)
    assert_matmul_close(out[rows], r64["out"], r32["out"], what="C5 full, sampled rows")
    # without the residual X, which would hide an error in the K = 8192 product
    x = u["X"][rows].astype(np.float64)
    assert_matmul_close(out[rows] - x, r64["out"] - x, r32["out"] - x, what="C5 full, out - X")
    # the GELU-gated intermediate (K = 2048 products) on the same rows
    if "U" in res.env:
        assert_matmul_close(res.env["U"][rows], r64["U"], r32["U"], what="C5 full U")
