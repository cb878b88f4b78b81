"""Degenerate and ragged shapes through every strategy on the GPU, against the fp64
oracle: single rows / columns / elements, K = 1 matmuls, one-column reductions,
softmax over one column, odd sizes that leave partial vector chunks, and non-finite
values flowing through elementwise chains and reductions."""

from __future__ import annotations

import numpy as np
import pytest

from metellus_b200 import Operations, run
from oracle.ir_eval import evaluate
from tests.tolerances import assert_elementwise_close, assert_matmul_close

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,K,N", [(1, 1, 1), (1, 64, 1), (7, 1, 9), (1, 300, 257), (129, 33, 1), (3, 5, 7)])
def test_matmul_tiny_and_ragged(cuda_device, M, K, N):
    r = np.random.default_rng(M * 100 + K * 10 + N)
    ops = Operations()
    ops.from_numpy(r.normal(0, 1, (M, K)).astype(np.float32), "A")
    ops.from_numpy(r.normal(0, 1, (K, N)).astype(np.float32), "B")
    ops.matmul(a="A", b="B", out="C")
    res = run(ops)
    r64, r32 = evaluate(ops, np.float64), evaluate(ops, np.float32)
    assert_matmul_close(res.env["C"], r64["C"], r32["C"], what=f"{M}x{K}x{N}")


@pytest.mark.parametrize("shape", [(1, 1), (1, 7), (5, 1), (3, 1027), (1027, 3)])
def test_elementwise_dag_odd_shapes(cuda_device, shape):
    r = np.random.default_rng(sum(shape))
    ops = Operations()
    for n in ("x", "y"):
        ops.from_numpy(r.uniform(-2, 2, shape).astype(np.float32), n)
    ops.elementwise("mul", out="a", operands=("x", "y"))
    ops.elementwise("exp", out="e", operands=("x",))
    ops.elementwise("add", out="out", operands=("a", "e"))
    res = run(ops)
    ref = evaluate(ops, np.float64)["out"]
    assert_elementwise_close(res.env["out"], ref, what=f"dag {shape}")


@pytest.mark.parametrize("M,K", [(1, 1), (4, 1), (1, 4096), (3, 5), (257, 129)])
def test_softmax_odd_rows(cuda_device, M, K):
    r = np.random.default_rng(M + K)
    ops = Operations()
    ops.from_numpy(r.normal(0, 2, (M, K)).astype(np.float32), "X")
    ops.reduction("max", out="mx", x="X", axis=-1)
    ops.reshape("mx", (M, 1), out="mx2")
    ops.elementwise("subtract", out="sh", operands=("X", "mx2"), y_broadcast="col")
    ops.elementwise("exp", out="e", operands=("sh",))
    ops.reduction("sum", out="sm", x="e", axis=-1)
    ops.reshape("sm", (M, 1), out="sm2")
    ops.elementwise("div", out="p", operands=("e", "sm2"), y_broadcast="col")
    res = run(ops)
    ref = evaluate(ops, np.float64)["p"]
    assert_elementwise_close(res.env["p"], ref, what=f"softmax {M}x{K}")


@pytest.mark.parametrize("op", ["sum", "max", "min", "product"])
@pytest.mark.parametrize("M,K", [(5, 1), (1, 1), (33, 3)])
def test_reduction_tiny(cuda_device, op, M, K):
    r = np.random.default_rng(M * K)
    X = (1 + r.uniform(-0.1, 0.1, (M, K))).astype(np.float32)
    ops = Operations()
    ops.from_numpy(X, "X")
    ops.reduction(op, out="R", x="X", axis=-1)
    res = run(ops)
    ref = evaluate(ops, np.float64)["R"]
    assert_elementwise_close(res.env["R"], ref, what=f"{op} {M}x{K}")


def test_non_finite_values_propagate(cuda_device):
    """inf / nan through a chain and a reduction: same placement as the oracle."""
    X = np.array([[1.0, np.inf, -2.0, 0.0], [np.nan, 1.0, 2.0, 3.0], [-np.inf, -1.0, 0.5, 4.0]], np.float32)
    ops = Operations()
    ops.from_numpy(X, "X")
    ops.elementwise("mul", out="a", operands=("X", 2.0))
    ops.elementwise("max", out="b", operands=("a", 0.0))
    ops.reduction("sum", out="s", x="b", axis=-1)
    res = run(ops)
    ref = evaluate(ops, np.float32)
    np.testing.assert_array_equal(res.env["s"], ref["s"])   # row 0: inf; NaN dropped by max
    ops2 = Operations()
    ops2.from_numpy(X, "X")
    ops2.elementwise("mul", out="a", operands=("X", 2.0))
    ops2.elementwise("add", out="b", operands=("a", 1.0))
    res2 = run(ops2)
    np.testing.assert_array_equal(res2.env["b"], evaluate(ops2, np.float32)["b"])  # inf, nan kept


def test_row_fused_value_with_second_consumer(cuda_device):
    """A value the row pass fuses into a reduction's kernel but that another kernel
    also reads (here t0, read by the reduction and by the matmul prologue) must still
    be written to memory (found by the planner property test)."""
    r = np.random.default_rng(2220)
    ops = Operations()
    ops.from_numpy(r.normal(size=(64, 128)).astype(np.float32), "x0")
    ops.from_numpy(r.normal(size=(128, 64)).astype(np.float32), "W")
    ops.elementwise("max", out="t0", operands=("x0", "x0"))
    ops.reduction("max", out="r", x="t0", axis=-1)
    ops.reshape("r", (64, 1), out="rc")
    ops.elementwise("subtract", out="t1", operands=("t0", "rc"), y_broadcast="col")
    ops.matmul(a="t1", b="W", out="t3")
    res = run(ops)
    r64, r32 = evaluate(ops, np.float64), evaluate(ops, np.float32)
    assert_matmul_close(res.env["t3"], r64["t3"], r32["t3"], what="row-fused second consumer")


@pytest.mark.parametrize("kind", ["colsum", "symmetrise"])
def test_transposed_view_of_inner_product(cuda_device, kind):
    """t = exp(x) on a square x, then sum(transpose(t)) or t + transpose(t): the reads
    of the transposed view must see all of t (separate kernels), matching the oracle."""
    r = np.random.default_rng(21)
    ops = Operations()
    ops.from_numpy(r.normal(0, 1, (192, 192)).astype(np.float32), "x")
    ops.elementwise("exp", "t", ("x",))
    ops.transpose("t", out="tt")
    if kind == "colsum":
        ops.reduction("sum", out="y", x="tt")
    else:
        ops.elementwise("add", "y", ("t", "tt"))
    res = run(ops)
    ref = evaluate(ops, np.float64)["y"]
    np.testing.assert_allclose(res.env["y"], ref, rtol=2e-6, atol=0)
