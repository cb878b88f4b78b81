"""The five benchmark programs, built through the public ``Operations`` API.

Shapes, value distributions and decompositions are the benchmark configurations:
softmax follows the reference's primitive decomposition (sandbox.py:388-408),
layernorm and GELU-tanh the reference runner's (runner.py:311-339, 232-261). Each
builder takes the full-size shape by default and smaller shapes for tests; inputs are
seeded ``numpy.random.default_rng`` draws, generated as float32.

* C1 ``matmul_bias_relu``:   C = relu(A @ B + bias)
* C2 ``elementwise_dag``:    out = tanh(x*y + z)*0.5 + sigmoid(x) - max(z*0.25, x)
* C3 ``row_softmax``:        out = exp(X - rowmax X) / rowsum(exp(X - rowmax X))
  and ``tensor_sum``:        s = sum(X) (whole tensor, through a (1, M*K) view)
* C4 ``attention``:          O = softmax((Q @ K^T) * 0.125) @ V per batch
* C5 ``mlp``:                H = layernorm(X); U = gelu_tanh(H@W1 + b1) * (H@W3);
                             out = U@W2 + b2 + X
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable

import numpy as np

from metellus_b200.orchestrator.builder import Operations


def _rng(seed: int) -> np.random.Generator:
    return np.random.default_rng(seed)


class Shaped:
    """Shape-only stand-in for an input array (plans depend only on shapes)."""

    def __init__(self, shape: tuple[int, ...]) -> None:
        self.shape = tuple(shape)
        self.dtype = np.float32


def _draw(r, kind: str, a: float, b: float, shape, materialize: bool):
    if not materialize:
        return Shaped(shape)
    f = r.normal if kind == "normal" else r.uniform
    return f(a, b, shape).astype(np.float32)


def _declare(ops: Operations, name: str, arr) -> None:
    if isinstance(arr, Shaped):
        ops.input(name, arr.shape)
    else:
        ops.from_numpy(arr, name)


def matmul_bias_relu(M: int = 1024, K: int = 1024, N: int = 1024, seed: int = 0,
                     materialize: bool = True) -> Operations:
    r = _rng(seed)
    A = _draw(r, "normal", 0.0, 1.0 / math.sqrt(K), (M, K), materialize)
    B = _draw(r, "normal", 0.0, 1.0 / math.sqrt(K), (K, N), materialize)
    bias = _draw(r, "normal", 0.0, 1.0, (1, N), materialize)
    ops = Operations()
    _declare(ops, "A", A)
    _declare(ops, "B", B)
    _declare(ops, "bias", bias)
    ops.matmul(a="A", b="B", out="C0")
    ops.elementwise("add", out="Cb", operands=("C0", "bias"), y_broadcast="row")
    ops.elementwise("max", out="C", operands=("Cb", 0.0))
    return ops


def elementwise_dag(M: int = 8192, N: int = 8192, seed: int = 0, materialize: bool = True) -> Operations:
    r = _rng(seed)
    x = _draw(r, "uniform", -1.0, 1.0, (M, N), materialize)
    y = _draw(r, "uniform", -1.0, 1.0, (M, N), materialize)
    z = _draw(r, "uniform", -1.0, 1.0, (M, N), materialize)
    return elementwise_dag_ops(x, y, z)


def elementwise_dag_ops(x, y, z) -> Operations:
    ops = Operations()
    _declare(ops, "x", x)
    _declare(ops, "y", y)
    _declare(ops, "z", z)
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
    return ops


def row_softmax(M: int = 32768, K: int = 4096, seed: int = 0, X=None, materialize: bool = True) -> Operations:
    if X is None:
        X = _draw(_rng(seed), "normal", 0.0, 2.0, (M, K), materialize)
    M, K = X.shape
    ops = Operations()
    _declare(ops, "X", X)
    ops.reduction("max", out="row_max_1d", x="X", axis=-1)
    ops.reshape("row_max_1d", (M, 1), out="row_max")
    ops.elementwise("subtract", out="shifted", operands=("X", "row_max"), y_broadcast="col")
    ops.elementwise("exp", out="e", operands=("shifted",))
    ops.reduction("sum", out="row_sum_1d", x="e", axis=-1)
    ops.reshape("row_sum_1d", (M, 1), out="row_sum")
    ops.elementwise("div", out="probs", operands=("e", "row_sum"), y_broadcast="col")
    return ops


def tensor_sum(M: int = 32768, K: int = 4096, seed: int = 0, X=None, materialize: bool = True) -> Operations:
    if X is None:
        X = _draw(_rng(seed), "normal", 0.0, 2.0, (M, K), materialize)
    M, K = X.shape
    ops = Operations()
    _declare(ops, "X", X)
    ops.reshape("X", (1, M * K), out="X_flat")
    ops.reduction("sum", out="total", x="X_flat", axis=-1)
    return ops


def attention(B: int = 128, S: int = 1024, D: int = 64, seed: int = 0, materialize: bool = True) -> Operations:
    r = _rng(seed)
    Q = _draw(r, "normal", 0.0, 1.0, (B, S, D), materialize)
    K = _draw(r, "normal", 0.0, 1.0, (B, S, D), materialize)
    V = _draw(r, "normal", 0.0, 1.0, (B, S, D), materialize)
    return attention_ops(Q, K, V)


def attention_ops(Q, K, V, scale: float = 0.125) -> Operations:
    B, S, _ = Q.shape
    ops = Operations()
    _declare(ops, "Q", Q)
    _declare(ops, "K", K)
    _declare(ops, "V", V)
    ops.transpose("K", out="Kt")
    ops.matmul(a="Q", b="Kt", out="scores")
    ops.elementwise("mul", out="scaled", operands=("scores", scale))
    ops.reduction("max", out="row_max_1d", x="scaled", axis=-1)
    ops.reshape("row_max_1d", (B, S, 1), out="row_max")
    ops.elementwise("subtract", out="shifted", operands=("scaled", "row_max"), y_broadcast="col")
    ops.elementwise("exp", out="e", operands=("shifted",))
    ops.reduction("sum", out="row_sum_1d", x="e", axis=-1)
    ops.reshape("row_sum_1d", (B, S, 1), out="row_sum")
    ops.elementwise("div", out="probs", operands=("e", "row_sum"), y_broadcast="col")
    ops.matmul(a="probs", b="V", out="O")
    return ops


def mlp(M: int = 16384, D: int = 2048, F: int = 8192, seed: int = 0, materialize: bool = True) -> Operations:
    r = _rng(seed)
    X = _draw(r, "normal", 0.0, 1.0, (M, D), materialize)
    W1 = _draw(r, "normal", 0.0, 1.0 / math.sqrt(D), (D, F), materialize)
    W3 = _draw(r, "normal", 0.0, 1.0 / math.sqrt(D), (D, F), materialize)
    W2 = _draw(r, "normal", 0.0, 1.0 / math.sqrt(F), (F, D), materialize)
    b1 = _draw(r, "normal", 0.0, 0.02, (1, F), materialize)
    b2 = _draw(r, "normal", 0.0, 0.02, (1, D), materialize)
    return mlp_ops(X, W1, W3, W2, b1, b2)


def mlp_ops(X, W1, W3, W2, b1, b2, eps: float = 1e-5) -> Operations:
    M, D = X.shape
    ops = Operations()
    for name, a in (("X", X), ("W1", W1), ("W3", W3), ("W2", W2), ("b1", b1), ("b2", b2)):
        _declare(ops, name, a)
    # layernorm (gamma = 1, beta = 0): runner.py:311-339
    ops.reduction("sum", out="row_sum", x="X", axis=-1)
    ops.elementwise("mul", out="mean", operands=("row_sum", 1.0 / D))
    ops.reshape("mean", (M, 1), out="mean_2d")
    ops.elementwise("subtract", out="centered", operands=("X", "mean_2d"), y_broadcast="col")
    ops.elementwise("mul", out="sq", operands=("centered", "centered"))
    ops.reduction("sum", out="sq_sum", x="sq", axis=-1)
    ops.elementwise("mul", out="var", operands=("sq_sum", 1.0 / D))
    ops.elementwise("add", out="var_eps", operands=("var", eps))
    ops.elementwise("sqrt", out="std", operands=("var_eps",))
    ops.reshape("std", (M, 1), out="std_2d")
    ops.elementwise("div", out="H", operands=("centered", "std_2d"), y_broadcast="col")
    # up projections and GELU-tanh: runner.py:232-261
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
    return ops


@dataclass(frozen=True)
class Config:
    key: str
    build: Callable[..., Operations]
    full: dict
    small: dict
    bound: str          # "hbm" | "tensor" | "fma"
    output: str


CONFIGS = {
    "c1": Config("c1", matmul_bias_relu, dict(M=1024, K=1024, N=1024), dict(M=256, K=192, N=320), "tensor", "C"),
    "c2": Config("c2", elementwise_dag, dict(M=8192, N=8192), dict(M=512, N=768), "hbm", "out"),
    "c3": Config("c3", row_softmax, dict(M=32768, K=4096), dict(M=512, K=4096), "hbm", "probs"),
    "c3sum": Config("c3sum", tensor_sum, dict(M=32768, K=4096), dict(M=512, K=1024), "hbm", "total"),
    "c4": Config("c4", attention, dict(B=128, S=1024, D=64), dict(B=4, S=256, D=64), "tensor", "O"),
    "c5": Config("c5", mlp, dict(M=16384, D=2048, F=8192), dict(M=256, D=256, F=512), "tensor", "out"),
}


def algorithmic_work(key: str, **shape) -> tuple[float, float]:
    """(flops, bytes) of one run of config ``key`` at ``shape`` — the roofline
    numerators (bytes = every input read once + every program output written once)."""
    s = {**CONFIGS[key].full, **shape}
    if key == "c1":
        M, K, N = s["M"], s["K"], s["N"]
        return 2.0 * M * N * K, 4.0 * (M * K + K * N + N + M * N)
    if key == "c2":
        n = s["M"] * s["N"]
        return 0.0, 4.0 * 4 * n
    if key == "c3":
        n = s["M"] * s["K"]
        return 0.0, 4.0 * 2 * n
    if key == "c3sum":
        return 0.0, 4.0 * s["M"] * s["K"]
    if key == "c4":
        B, S, D = s["B"], s["S"], s["D"]
        return B * 2.0 * (2.0 * S * S * D), 4.0 * 4 * B * S * D
    if key == "c5":
        M, D, F = s["M"], s["D"], s["F"]
        return 3 * 2.0 * M * D * F, 4.0 * (2 * M * D + 3 * D * F + F + D)
    raise KeyError(key)


SHARD_AXIS = {"c1": None, "c2": "M", "c3": "M", "c3sum": "M", "c4": "B", "c5": "M"}


def shard(key: str, world: int, rank: int, seed: int = 0, **shape) -> tuple[Operations, dict]:
    """Rank ``rank``'s part of config ``key`` split ``world`` ways (strong scaling).

    The full configuration's inputs are drawn (seeded, identical on every rank) and the
    program is rebuilt on this rank's contiguous block of rows (C2, C3, C3-sum, C5) or
    heads (C4); weights (C5's W1, W3, W2 and biases) are replicated. C1 has no batch or
    row dimension to split (its 1024 rows are one GEMM), so every rank runs the whole
    program (replicas). Returns (ops, this rank's shape)."""
    from metellus_b200.distributed import row_range

    c = CONFIGS[key]
    full = {**c.full, **shape}
    axis = SHARD_AXIS[key]
    if axis is None or world == 1:
        return c.build(**full, seed=seed), full
    a, b = row_range(full[axis], rank, world)
    u = c.build(**full, seed=seed).uploads
    local = {**full, axis: b - a}
    if key == "c2":
        return elementwise_dag_ops(u["x"][a:b], u["y"][a:b], u["z"][a:b]), local
    if key == "c3":
        return row_softmax(X=u["X"][a:b]), local
    if key == "c3sum":
        return tensor_sum(X=u["X"][a:b]), local
    if key == "c4":
        return attention_ops(u["Q"][a:b], u["K"][a:b], u["V"][a:b]), local
    if key == "c5":
        return mlp_ops(u["X"][a:b], u["W1"], u["W3"], u["W2"], u["b1"], u["b2"]), local
    raise KeyError(key)
