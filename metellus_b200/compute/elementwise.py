"""Elementwise op table: names, arity and the CUDA C++ expression of each op.

The op *names*, arities, broadcast modes and value semantics are the reference's
(src/compute/elementwise/elementwise.py:18-57); the expressions are CUDA C++ written
for sm_100a:

* add / subtract / mul / div / recip use the ``__f*_rn`` intrinsics so that nvcc /
  NVRTC never contracts ``x*y+z`` into an FMA. A chain of add/mul/max/select ops is
  therefore bit-identical to the same chain evaluated in IEEE fp32 on the host.
* ``tanh`` calls CUDA's ``tanhf`` (saturates cleanly to +-1 at +-inf). The
  reference spells tanh as ``copysign(1 - 2/(1 + exp(2|x|)), x)`` only to dodge a
  Metal overflow bug (elementwise.py:28-32); that form loses all relative accuracy
  near 0, so it is not reproduced on the device.
* comparisons produce 1.0f / 0.0f (expressions.py:43-48); ``max``/``min`` are the
  NaN-dropping ``fmaxf``/``fminf`` (C ``fmax``/``fmin`` semantics, as MSL's).
"""

from __future__ import annotations

from enum import StrEnum


class BroadcastSpec(StrEnum):
    """How a secondary operand maps onto the primary's (M, N) matrix."""

    NONE = "none"
    SCALAR = "scalar"
    ROW = "row"
    COL = "col"


UNARY_EXPRESSIONS = {
    "negate": "(-x)",
    "absolute": "fabsf(x)",
    "exp": "expf(x)",
    "log": "logf(x)",
    "sqrt": "sqrtf(x)",
    "recip": "__fdiv_rn(1.0f, x)",
    "sin": "sinf(x)",
    "cos": "cosf(x)",
    "tanh": "tanhf(x)",
    "floor": "floorf(x)",
    "ceil": "ceilf(x)",
    "sign": "((x > 0.0f) ? 1.0f : ((x < 0.0f) ? -1.0f : 0.0f))",
}

BINARY_EXPRESSIONS = {
    "add": "__fadd_rn(x, y)",
    "subtract": "__fsub_rn(x, y)",
    "mul": "__fmul_rn(x, y)",
    "div": "__fdiv_rn(x, y)",
    "max": "fmaxf(x, y)",
    "min": "fminf(x, y)",
    "pow": "powf(x, y)",
    "equal": "x == y",
    "not_equal": "x != y",
    "lt": "x < y",
    "gt": "x > y",
    "ge": "x >= y",
    "le": "x <= y",
}

TERNARY_EXPRESSIONS = {
    "where": "((cond != 0.0f) ? x : y)",
}

COMPARISON_OPS = frozenset({"equal", "not_equal", "lt", "gt", "ge", "le"})
BROADCAST_MODES = frozenset(m.value for m in BroadcastSpec)

# Ops whose device result is exactly the IEEE fp32 result of the host formula.
EXACT_OPS = frozenset(
    {"negate", "absolute", "recip", "sqrt", "floor", "ceil", "sign", "add", "subtract",
     "mul", "div", "max", "min", "where"} | COMPARISON_OPS
)


def supported_elementwise_ops() -> tuple[str, ...]:
    return tuple(sorted((*UNARY_EXPRESSIONS, *BINARY_EXPRESSIONS, *TERNARY_EXPRESSIONS)))


def elementwise_arity(op: str) -> int:
    if op in UNARY_EXPRESSIONS:
        return 1
    if op in BINARY_EXPRESSIONS:
        return 2
    if op in TERNARY_EXPRESSIONS:
        return 3
    raise ValueError(
        f"Unsupported elementwise op {op!r}; expected one of {supported_elementwise_ops()}"
    )


def elementwise_expression(op: str) -> str:
    for table in (UNARY_EXPRESSIONS, BINARY_EXPRESSIONS, TERNARY_EXPRESSIONS):
        if op in table:
            return table[op]
    raise ValueError(
        f"Unsupported elementwise op {op!r}; expected one of {supported_elementwise_ops()}"
    )


def elementwise_outputs_bool(op: str) -> bool:
    elementwise_expression(op)
    return op in COMPARISON_OPS
