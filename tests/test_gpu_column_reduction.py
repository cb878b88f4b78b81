"""GPU parity of the column-reduction kernel: a last-axis reduction over a view whose
rows are contiguous, ``reduction(transpose(X))`` (the reference reduces a row-major
matrix over its first axis this way, sandbox.py:177-186), with and without prologue /
epilogue chains, against the oracle. Ragged output counts (not a multiple of 4 or
of the 128-output block), shallow and deep reduced axes (one split and many splits),
and repeated launches of one plan (the split tickets reset themselves)."""

from __future__ import annotations

import numpy as np
import pytest

from metellus_b200 import Executable, Operations, run
from oracle.ir_eval import evaluate

pytestmark = pytest.mark.gpu


def _program(X, op, *, pro=None, epi=None):
    ops = Operations()
    ops.from_numpy(X, "X")
    ops.transpose("X", out="Xt")
    src = "Xt"
    if pro:
        ops.elementwise(pro[0], "P", (src, *pro[1:]))
        src = "P"
    ops.reduction(op, out="R", x=src)
    if epi:
        ops.elementwise(epi[0], "E", ("R", *epi[1:]))
    return ops


def _check(ops, out, res_env, op):
    ref = evaluate(ops, np.float64)[out]
    got = res_env[out].astype(np.float64)
    x = ops.uploads["X"].astype(np.float64)
    if op in ("max", "min"):
        np.testing.assert_array_equal(res_env[out], np.float32(ref))
        return
    ulp = np.spacing(np.abs(np.float32(ref))).astype(np.float64)
    if op == "sum":
        tol = 2e-6 * np.abs(x).sum(axis=0) + ulp
    else:  # fp32 product: each of the K roundings perturbs the result by <= 2^-24 relative
        tol = 10 * np.sqrt(x.shape[0]) * 2.0 ** -24 * np.abs(ref) + ulp
    assert np.all(np.abs(got - ref) <= tol), np.max(np.abs(got - ref) / tol)


def _uses_column_kernel(res):
    names = [g.kernel.function_name for g in res.groups]
    assert any(n.startswith("reduce_cols_") for n in names), names


@pytest.mark.parametrize("op", ["sum", "max", "min", "product"])
@pytest.mark.parametrize("shape", [(4096, 1024), (1000, 333), (37, 130), (200_000, 12), (64, 8192), (3, 5)])
def test_column_reduction(cuda_device, op, shape):
    r = np.random.default_rng(11)
    X = (1.0 + r.uniform(-1e-3, 1e-3, shape)).astype(np.float32) if op == "product" else \
        r.normal(0, 1, shape).astype(np.float32)
    ops = _program(X, op)
    res = run(ops)
    _uses_column_kernel(res)
    _check(ops, "R", res.env, op)


def test_column_reduction_prologue_epilogue(cuda_device):
    r = np.random.default_rng(12)
    X = r.normal(0, 1, (3000, 777)).astype(np.float32)
    ops = _program(X, "sum", pro=("exp",), epi=("mul", 1.0 / 3000))
    res = run(ops)
    _uses_column_kernel(res)
    ref = evaluate(ops, np.float64)["E"]
    scale = np.exp(X.astype(np.float64)).sum(axis=0) / 3000
    assert np.all(np.abs(res.env["E"] - ref) <= 4e-6 * scale)


def test_column_reduction_repeated(cuda_device):
    """One plan launched many times (graph replay): the per-column-block tickets are
    reset by the last split block, so every replay combines its own partials."""
    r = np.random.default_rng(13)
    X = r.normal(0, 1, (8192, 640)).astype(np.float32)
    ops = _program(X, "sum")
    exe = Executable(ops, outputs=("R",))
    for i in range(4):
        Xi = (X + i).astype(np.float32)
        got = exe({"X": Xi})["R"].astype(np.float64)
        ref = Xi.astype(np.float64).sum(axis=0)
        assert np.all(np.abs(got - ref) <= 2e-6 * np.abs(Xi.astype(np.float64)).sum(axis=0) + 1e-6)
    exe.close()
