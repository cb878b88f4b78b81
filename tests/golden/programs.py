"""Program specs shared by the golden-fixture generator and the plan tests.

Each spec is a function ``spec(ops)`` that declares inputs with ``ops.input`` and
appends ops through the builder methods both the reference's ``Operations`` and
``metellus_b200.Operations`` expose (input / matmul / elementwise / reduction /
transpose / reshape), so the same program can be replayed into either fuser."""

from __future__ import annotations

import math


def c1(ops, M=256, K=192, N=320):
    ops.input("A", (M, K))
    ops.input("B", (K, N))
    ops.input("bias", (1, N))
    ops.matmul(a="A", b="B", out="C0")
    ops.elementwise("add", out="Cb", operands=("C0", "bias"), y_broadcast="row")
    ops.elementwise("max", out="C", operands=("Cb", 0.0))


def c2(ops, M=512, N=768):
    for n in ("x", "y", "z"):
        ops.input(n, (M, N))
    ops.elementwise("mul", out="xy", operands=("x", "y"))
    ops.elementwise("add", out="xyz", operands=("xy", "z"))
    ops.elementwise("tanh", out="th", operands=("xyz",))
    ops.elementwise("mul", out="t", operands=("th", 0.5))
    ops.elementwise("negate", out="nx", operands=("x",))
    ops.elementwise("exp", out="enx", operands=("nx",))
    ops.elementwise("add", out="den", operands=("enx", 1.0))
    ops.elementwise("recip", out="s", operands=("den",))
    ops.elementwise("mul", out="zq", operands=("z", 0.25))
    ops.elementwise("max", out="m", operands=("zq", "x"))
    ops.elementwise("add", out="ts", operands=("t", "s"))
    ops.elementwise("subtract", out="out", operands=("ts", "m"))


def c3(ops, M=512, K=4096):
    ops.input("X", (M, K))
    ops.reduction("max", out="row_max_1d", x="X", axis=-1)
    ops.reshape("row_max_1d", (M, 1), out="row_max")
    ops.elementwise("subtract", out="shifted", operands=("X", "row_max"), y_broadcast="col")
    ops.elementwise("exp", out="e", operands=("shifted",))
    ops.reduction("sum", out="row_sum_1d", x="e", axis=-1)
    ops.reshape("row_sum_1d", (M, 1), out="row_sum")
    ops.elementwise("div", out="probs", operands=("e", "row_sum"), y_broadcast="col")


def c3sum(ops, M=512, K=1024):
    ops.input("X", (M, K))
    ops.reshape("X", (1, M * K), out="X_flat")
    ops.reduction("sum", out="total", x="X_flat", axis=-1)


def c4_head(ops, S=256, D=64):
    """One attention head (the reference IR is rank 2; the batched program repeats
    this plan per batch index)."""
    ops.input("Q", (S, D))
    ops.input("K", (S, D))
    ops.input("V", (S, D))
    ops.transpose("K", out="Kt")
    ops.matmul(a="Q", b="Kt", out="scores")
    ops.elementwise("mul", out="scaled", operands=("scores", 0.125))
    ops.reduction("max", out="row_max_1d", x="scaled", axis=-1)
    ops.reshape("row_max_1d", (S, 1), out="row_max")
    ops.elementwise("subtract", out="shifted", operands=("scaled", "row_max"), y_broadcast="col")
    ops.elementwise("exp", out="e", operands=("shifted",))
    ops.reduction("sum", out="row_sum_1d", x="e", axis=-1)
    ops.reshape("row_sum_1d", (S, 1), out="row_sum")
    ops.elementwise("div", out="probs", operands=("e", "row_sum"), y_broadcast="col")
    ops.matmul(a="probs", b="V", out="O")


def c5(ops, M=256, D=256, F=512):
    for n, s in (("X", (M, D)), ("W1", (D, F)), ("W3", (D, F)), ("W2", (F, D)), ("b1", (1, F)),
                 ("b2", (1, D))):
        ops.input(n, s)
    ops.reduction("sum", out="row_sum", x="X", axis=-1)
    ops.elementwise("mul", out="mean", operands=("row_sum", 1.0 / D))
    ops.reshape("mean", (M, 1), out="mean_2d")
    ops.elementwise("subtract", out="centered", operands=("X", "mean_2d"), y_broadcast="col")
    ops.elementwise("mul", out="sq", operands=("centered", "centered"))
    ops.reduction("sum", out="sq_sum", x="sq", axis=-1)
    ops.elementwise("mul", out="var", operands=("sq_sum", 1.0 / D))
    ops.elementwise("add", out="var_eps", operands=("var", 1e-5))
    ops.elementwise("sqrt", out="std", operands=("var_eps",))
    ops.reshape("std", (M, 1), out="std_2d")
    ops.elementwise("div", out="H", operands=("centered", "std_2d"), y_broadcast="col")
    ops.matmul(a="H", b="W1", out="z1")
    ops.elementwise("add", out="z1b", operands=("z1", "b1"), y_broadcast="row")
    ops.elementwise("mul", out="g_sq", operands=("z1b", "z1b"))
    ops.elementwise("mul", out="g_cu", operands=("g_sq", "z1b"))
    ops.elementwise("mul", out="g_c", operands=("g_cu", 0.044715))
    ops.elementwise("add", out="g_s", operands=("z1b", "g_c"))
    ops.elementwise("mul", out="g_k", operands=("g_s", math.sqrt(2.0 / math.pi)))
    ops.elementwise("tanh", out="g_t", operands=("g_k",))
    ops.elementwise("add", out="g_1", operands=("g_t", 1.0))
    ops.elementwise("mul", out="g_h", operands=("z1b", 0.5))
    ops.elementwise("mul", out="gelu", operands=("g_h", "g_1"))
    ops.matmul(a="H", b="W3", out="z3")
    ops.elementwise("mul", out="U", operands=("gelu", "z3"))
    ops.matmul(a="U", b="W2", out="z2")
    ops.elementwise("add", out="z2b", operands=("z2", "b2"), y_broadcast="row")
    ops.elementwise("add", out="out", operands=("z2b", "X"))


# -- shapes exercised by the reference's own fusion tests (tests/test_fusion.py) -------


def relu_matmul_bias(ops):
    ops.input("A", (32, 64))
    ops.input("B", (64, 128))
    ops.input("bias", (1, 128))
    ops.matmul(a="A", b="B", out="C")
    ops.elementwise("add", out="Cb", operands=("C", "bias"), y_broadcast="row")
    ops.elementwise("max", out="Y", operands=("Cb", 0.0))


def relu_matmul(ops):
    ops.input("A", (32, 64))
    ops.input("B", (64, 48))
    ops.matmul(a="A", b="B", out="C")
    ops.elementwise("max", out="D", operands=("C", 0.0))


def prologue_on_a(ops):
    ops.input("A", (32, 64))
    ops.input("B", (64, 48))
    ops.elementwise("max", out="Ar", operands=("A", 0.0))
    ops.matmul(a="Ar", b="B", out="C")


def prologue_reduction(ops):
    ops.input("X", (64, 96))
    ops.elementwise("exp", out="E", operands=("X",))
    ops.reduction("sum", out="S", x="E", axis=-1)


def reduction_epilogue(ops):
    ops.input("X", (64, 96))
    ops.reduction("sum", out="S", x="X", axis=-1)
    ops.elementwise("mul", out="T", operands=("S", 0.5))


def multi_consumer_matmul(ops):
    ops.input("A", (32, 16))
    ops.input("B", (16, 24))
    ops.matmul(a="A", b="B", out="C")
    ops.elementwise("max", out="D", operands=("C", 0.0))
    ops.elementwise("absolute", out="E", operands=("C",))


def upstream_recompute(ops):
    ops.input("X", (32, 64))
    ops.input("B1", (64, 48))
    ops.input("B2", (64, 40))
    ops.elementwise("max", out="X1", operands=("X", 0.0))
    ops.matmul(a="X1", b="B1", out="t1")
    ops.matmul(a="X1", b="B2", out="t2")


def multi_producer(ops):
    for n, s in (("A", (32, 64)), ("B", (64, 48)), ("C", (32, 80)), ("D", (80, 48))):
        ops.input(n, s)
    ops.matmul(a="A", b="B", out="c1")
    ops.matmul(a="C", b="D", out="c2")
    ops.elementwise("add", out="z", operands=("c1", "c2"))


def diamond(ops):
    for n, s in (("A", (32, 64)), ("B1", (64, 48)), ("B2", (64, 48))):
        ops.input(n, s)
    ops.matmul(a="A", b="B1", out="c1")
    ops.matmul(a="A", b="B2", out="c2")
    ops.elementwise("mul", out="z", operands=("c1", "c2"))


def where_standalone(ops):
    for n in ("X", "Y", "Cond"):
        ops.input(n, (24, 40))
    ops.elementwise("where", out="Z", operands=("X", "Y", "Cond"))


def overflow_multi_producer(ops):
    for n in ("A", "B", "C", "D"):
        ops.input(n, (64, 64))
    ops.matmul(a="A", b="B", out="c1")
    ops.matmul(a="C", b="D", out="c2")
    ops.elementwise("add", out="z", operands=("c1", "c2"))


def transposed_reduction(ops):
    """Reduction over the first axis, spelled as in the reference's sandbox
    (sandbox.py:177-186): the last axis of a transposed view."""
    ops.input("X", (96, 48))
    ops.transpose("X", out="Xt")
    ops.reduction("sum", out="S", x="Xt", axis=-1)


def transposed_reduction_chain(ops):
    ops.input("X", (96, 48))
    ops.transpose("X", out="Xt")
    ops.elementwise("exp", out="E", operands=("Xt",))
    ops.reduction("max", out="S", x="E", axis=-1)
    ops.elementwise("mul", out="T", operands=("S", 0.5))


PROGRAMS = {
    "c1": c1, "c2": c2, "c3": c3, "c3sum": c3sum, "c4_head": c4_head, "c5": c5,
    "relu_matmul_bias": relu_matmul_bias, "relu_matmul": relu_matmul, "prologue_on_a": prologue_on_a,
    "prologue_reduction": prologue_reduction, "reduction_epilogue": reduction_epilogue,
    "multi_consumer_matmul": multi_consumer_matmul, "upstream_recompute": upstream_recompute,
    "multi_producer": multi_producer, "diamond": diamond, "where_standalone": where_standalone,
    "overflow_multi_producer": overflow_multi_producer,
    "transposed_reduction": transposed_reduction, "transposed_reduction_chain": transposed_reduction_chain,
}
