"""Property tests of the planner on random programs (CPU only: plans and generated
source, no launches). For seeded random mixes of elementwise chains and DAGs,
row / column broadcasts, last-axis reductions with views (including first-axis
reductions through a transposed view), matmuls and diamonds:

* every op lands in exactly one kernel group, and the groups' ops in dispatch order
  respect every producer -> consumer edge of the program;
* a tensor read by a later group than its producer is materialised (bound) by the
  producing group;
* the B200 plan never needs more kernels than the reference pass set alone;
* the scheduler accepts the plan and every group renders CUDA source.
"""

from __future__ import annotations

import numpy as np
from hypothesis import given, settings
from hypothesis import strategies as st

from metellus_b200 import Operations
from metellus_b200.api.run import compile_program
from metellus_b200.orchestrator.scheduler import schedule

UNARY = ("negate", "exp", "tanh", "absolute", "sqrt", "recip")
BINARY = ("add", "subtract", "mul", "max", "min")


def random_program(seed: int, safe: bool = False, large: bool = False) -> Operations:
    """A seeded random program; ``safe`` keeps values finite and O(1) (no exp / sqrt /
    recip, sums instead of maxima) for numeric checks on the GPU; ``large`` picks
    shapes big enough for the tensor-core (tcgen05) plans."""
    r = np.random.default_rng(seed)
    unary = ("negate", "tanh", "absolute") if safe else UNARY
    if large:
        M = int(r.choice([128, 256, 384]))
        N = int(r.choice([128, 256]))
        P = int(r.choice([128, 256]))
    else:
        M = int(r.choice([32, 64, 96]))
        N = int(r.choice([32, 64, 128]))
        P = int(r.choice([32, 64]))
    ops = Operations()
    mats = []          # names of (M, N) tensors
    others = {}        # (M, P) tensors by name
    for i in range(int(r.integers(2, 4))):
        ops.from_numpy(r.normal(size=(M, N)).astype(np.float32), f"x{i}")
        # weights scaled 1 / sqrt(fan-in) so chained products stay O(1)
        mats.append(f"x{i}")
    shapes = {"bias": (1, N), "W": (N, P), "W2": (N, P), "WT": (P, N)}

    def need(name: str) -> str:  # inputs are declared on first use (every upload must be read)
        if name not in ops.tensors:
            scale = shapes[name][0] ** -0.5 if name in ("W", "W2") else shapes[name][1] ** -0.5 if name == "WT" else 1.0
            ops.from_numpy((scale * r.normal(size=shapes[name])).astype(np.float32), name)
        return name
    for k in range(int(r.integers(3, 11))):
        kind = r.choice(["unary", "binary", "scalar", "rowb", "softmaxish", "matmul", "diamond", "gated", "onp",
                         "tmatmul", "colred"],
                        p=[0.13, 0.14, 0.11, 0.08, 0.11, 0.08, 0.08, 0.1, 0.06, 0.05, 0.06])
        out = f"t{k}"
        if kind == "unary":
            ops.elementwise(str(r.choice(unary)), out=out, operands=(str(r.choice(mats)),))
            mats.append(out)
        elif kind == "binary":
            a, b = r.choice(mats, 2)
            ops.elementwise(str(r.choice(BINARY)), out=out, operands=(str(a), str(b)))
            mats.append(out)
        elif kind == "scalar":
            ops.elementwise(str(r.choice(BINARY)), out=out, operands=(str(r.choice(mats)), float(r.normal())))
            mats.append(out)
        elif kind == "rowb":
            ops.elementwise("add", out=out, operands=(str(r.choice(mats)), need("bias")), y_broadcast="row")
            mats.append(out)
        elif kind == "softmaxish":
            src = str(r.choice(mats))
            ops.reduction(str(r.choice(["max", "min"] if safe else ["max", "sum"])), out=f"{out}_r", x=src, axis=-1)
            ops.reshape(f"{out}_r", (M, 1), out=f"{out}_c")
            ops.elementwise("subtract", out=out, operands=(src, f"{out}_c"), y_broadcast="col")
            mats.append(out)
        elif kind == "matmul":
            ops.matmul(a=str(r.choice(mats)), b=need("W"), out=out)
            others[out] = (M, P)
        elif kind == "diamond":
            src = str(r.choice(mats))
            ops.matmul(a=src, b=need("W"), out=f"{out}_a")
            ops.matmul(a=src, b=need("W2"), out=f"{out}_b")
            ops.elementwise("mul", out=out, operands=(f"{out}_a", f"{out}_b"))
            others[out] = (M, P)
        elif kind == "gated":  # act(src @ W + c) * (src @ W2): the dual-GEMM epilogue shape
            src = str(r.choice(mats))
            ops.matmul(a=src, b=need("W"), out=f"{out}_a")
            ops.elementwise("add", out=f"{out}_c", operands=(f"{out}_a", 0.5))
            ops.elementwise("tanh", out=f"{out}_t", operands=(f"{out}_c",))
            ops.elementwise("mul", out=f"{out}_h", operands=(f"{out}_c", f"{out}_t"))
            ops.matmul(a=src, b=need("W2"), out=f"{out}_b")
            ops.elementwise("mul", out=out, operands=(f"{out}_h", f"{out}_b"))
            others[out] = (M, P)
        elif kind == "tmatmul":  # B as a transposed view of a (P, N) input
            if "WTt" not in ops.tensors:
                ops.transpose(need("WT"), out="WTt")
            ops.matmul(a=str(r.choice(mats)), b="WTt", out=out)
            others[out] = (M, P)
        elif kind == "colred" and M == N and r.random() < 0.5:  # square: add a transposed view
            src = str(r.choice(mats))
            ops.transpose(src, out=f"{out}_T")
            ops.elementwise("add", out=out, operands=(str(r.choice(mats)), f"{out}_T"))
            mats.append(out)
        elif kind == "colred":  # reduce over the first axis (a transposed view), add back as a row
            src = str(r.choice(mats))
            ops.transpose(src, out=f"{out}_T")
            ops.reduction(str(r.choice(["max", "min"] if safe else ["max", "sum"])), out=f"{out}_r", x=f"{out}_T",
                          axis=-1)
            ops.reshape(f"{out}_r", (1, N), out=f"{out}_row")
            ops.elementwise("add", out=out, operands=(str(r.choice(mats)), f"{out}_row"), y_broadcast="row")
            mats.append(out)
        elif others:  # an elementwise op over (M, P) results
            a = str(r.choice(list(others)))
            ops.elementwise(str(r.choice(unary)), out=out, operands=(a,))
            others[out] = (M, P)
    used = {t.buffer_key for op in ops.build() for t in op.inputs}
    for i, name in enumerate(n for n in list(ops.uploads) if n not in used):
        ops.elementwise("add", out=f"u{i}", operands=(name, mats[-1]))
    return ops


def _check_plan(ops: Operations, groups) -> None:
    program = ops.build()
    order = {id(op): i for i, op in enumerate(program)}
    where: dict[int, list[int]] = {}
    for gi, g in enumerate(groups):
        for op in g.ops:
            where.setdefault(id(op), []).append(gi)
    assert set(where) == set(order), "some ops were dropped"
    for op in program:
        if len(where[id(op)]) > 1:  # recompute: only elementwise prologues are replicated
            assert type(op).__name__ == "ElementwiseOp", f"{op.out.name} replicated"
    # the group that materialises each produced buffer (if any)
    materialised: dict[str, int] = {}
    for op in program:
        for gi in where[id(op)]:
            if op.out.buffer_key in groups[gi].bindings:
                materialised.setdefault(op.out.buffer_key, gi)
    produced = {op.out.buffer_key for op in program}
    for gi, g in enumerate(groups):
        local = {op.out.buffer_key for op in g.ops}
        for op in g.ops:
            for t in op.inputs:
                if t.buffer_key not in produced or t.buffer_key in local:
                    continue  # program input, or computed inside this group
                pg = materialised.get(t.buffer_key)
                assert pg is not None and pg < gi, \
                    f"{op.out.name} (group {gi}) reads {t.name}, materialised by group {pg}"


@settings(max_examples=200, deadline=None)
@given(st.integers(0, 10**6), st.booleans())
def test_random_programs_plan_soundly(seed, large):
    ops = random_program(seed, large=large)
    groups = compile_program(ops)
    _check_plan(ops, groups)
    ref_groups = compile_program(ops, b200=False)
    _check_plan(ops, ref_groups)
    assert len(groups) <= len(ref_groups)
    for g in groups:
        assert g.kernel.source  # renders
    runtime = schedule(ops, groups)
    assert len(runtime.fragments) > 0
