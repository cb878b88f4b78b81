"""The vertex graph treats view reads as edges to the view's storage owner (no GPU).

A vertex that reads a transposed / reshaped view depends on the owner's producer,
keeps it materialised and counts as its consumer; program outputs keep the
reference's definition (a tensor read only through a view is still an output)."""

from __future__ import annotations

import numpy as np

from metellus_b200 import Operations, compile_program
from metellus_b200.orchestrator.graph import Graph


def _program():
    ops = Operations()
    ops.from_numpy(np.ones((32, 48), np.float32), "x")
    ops.elementwise("exp", "t", ("x",))
    ops.transpose("t", out="tT")
    ops.reduction("sum", out="c", x="tT")          # column sums of t, through the view
    ops.reshape("c", (1, 48), out="c_row")
    ops.elementwise("add", "y", ("t", "c_row"), y_broadcast="row")
    return ops


def test_view_owner_map_and_reads():
    g = Graph.from_program(_program().build())
    assert g.view_owner == {"tT": "t", "c_row": "c"}
    red = next(v for v in g.vertices if v.ops[0].out.name == "c")
    assert g.reads(red) == {"tT", "t"}
    assert [v.ops[0].out.name for v in g.consumers_of("t")] == ["c", "y"]


def test_owner_of_a_view_stays_visible_and_ordered():
    g = Graph.from_program(_program().build())
    t = next(v for v in g.vertices if v.ops[0].out.name == "t")
    assert "t" in t.outputs
    order = [v.ops[0].out.name for v in g.topo_sort()]
    assert order.index("t") < order.index("c") < order.index("y")


def test_program_outputs_keep_the_reference_definition():
    ops = Operations()
    ops.from_numpy(np.ones((16, 8), np.float32), "x")
    ops.reduction("max", out="m", x="x")
    ops.reshape("m", (16, 1), out="m2")
    ops.elementwise("subtract", "y", ("x", "m2"), y_broadcast="col")
    g = Graph.from_program(ops.build())
    assert g.program_outputs == frozenset({"m", "y"})


def test_no_cycle_through_views():
    """t -> transpose -> column sum -> row-add into t's consumer: merging t's producer
    with that consumer would need the column sum both before and after it."""
    groups = compile_program(_program())
    names = [[op.out.name for op in g.ops] for g in groups]
    where = {n: i for i, ns in enumerate(names) for n in ns}
    assert where["t"] < where["c"] < where["y"]
