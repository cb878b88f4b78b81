"""Planner and codegen checks (no GPU) for reductions over views with contiguous rows,
``reduction(transpose(X))``: they get the coalesced column kernel, with the reduced
axis split across blocks only when the outputs alone do not fill the GPU, and the
rendered kernels compile for sm_100a."""

from __future__ import annotations

import numpy as np
import pytest

from metellus_b200 import Operations, compile_program
from metellus_b200.orchestrator.assembly.reduction import column_reduction_plan
from metellus_b200.runtime import backend
from oracle.ir_eval import evaluate


def _ops(R, C, *, pro=False, epi=False):
    ops = Operations()
    ops.from_numpy(np.ones((R, C), np.float32), "X")
    ops.transpose("X", out="Xt")
    src = "Xt"
    if pro:
        ops.elementwise("exp", "P", ("Xt",))
        src = "P"
    ops.reduction("sum", out="R", x=src)
    if epi:
        ops.elementwise("mul", "E", ("R", 0.5))
    return ops


@pytest.mark.parametrize("R,C,pro,epi", [(4096, 1024, False, False), (1000, 333, True, True), (64, 8192, False, True)])
def test_transposed_reduction_uses_column_kernel(R, C, pro, epi):
    groups = compile_program(_ops(R, C, pro=pro, epi=epi))
    assert len(groups) == 1
    g = groups[0]
    assert g.kernel.function_name.startswith("reduce_cols_")
    colblocks, splits = column_reduction_plan(C, R)
    assert g.grid == (colblocks, splits, 1)
    assert (len(g.scratch) == 2) == (splits > 1)
    backend.compile_cubin(g.kernel.source, name=g.kernel.function_name + ".cu")


def test_column_plan_fills_the_gpu():
    assert column_reduction_plan(1024, 4096) == (8, 64)        # 8 column blocks x 64 splits = 512
    assert column_reduction_plan(4096, 32768) == (32, 37)       # ~1184 blocks
    assert column_reduction_plan(200_000, 64) == (1563, 1)      # enough outputs: no split
    assert column_reduction_plan(12, 200_000) == (1, 1184)
    assert column_reduction_plan(5, 3) == (1, 1)


def test_row_major_reduction_keeps_row_templates():
    ops = Operations()
    ops.from_numpy(np.ones((64, 256), np.float32), "X")
    ops.reduction("sum", out="R", x="X")
    (g,) = compile_program(ops)
    assert not g.kernel.function_name.startswith("reduce_cols_")


def test_oracle_reads_transposed_views():
    X = np.arange(12, dtype=np.float32).reshape(3, 4)
    ops = Operations()
    ops.from_numpy(X, "X")
    ops.transpose("X", out="Xt")
    ops.reduction("sum", out="R", x="Xt")
    np.testing.assert_array_equal(evaluate(ops, np.float64)["R"], X.astype(np.float64).sum(axis=0))


def _square_transpose_programs():
    """Programs reading a transposed view of a tensor computed in the same program, on
    a square shape (the view has the owner's shape but swapped strides)."""
    out = {}
    ops = Operations()
    ops.from_numpy(np.arange(64 * 64, dtype=np.float32).reshape(64, 64) / 4096, "x")
    ops.elementwise("exp", "t", ("x",))
    ops.transpose("t", out="tt")
    ops.reduction("sum", out="s", x="tt")
    out["colsum"] = ops
    ops = Operations()
    ops.from_numpy(np.arange(64 * 64, dtype=np.float32).reshape(64, 64) / 4096, "x")
    ops.elementwise("exp", "t", ("x",))
    ops.transpose("t", out="tt")
    ops.elementwise("add", "y", ("t", "tt"))
    out["symmetrise"] = ops
    return out


@pytest.mark.parametrize("name", ["colsum", "symmetrise"])
def test_transposed_view_of_an_inner_product_is_not_fused(name):
    """A kernel that computes t element by element cannot also read transpose(t): the
    producer of t and the reader of its transposed view must be separate kernels (the
    reference's chain rule fuses ``t + transpose(t)`` and reads t before it is written)."""
    ops = _square_transpose_programs()[name]
    for g in compile_program(ops):
        names = {op.out.name for op in g.ops}
        for op in g.ops:
            for t in op.inputs:
                if t.name == "tt":
                    assert "t" not in names, (g.strategy, names)
