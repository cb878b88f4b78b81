"""CUDA expression building for elementwise chains (reference:
src/orchestrator/assembly/expressions.py:33-205).

``chain_value_transform`` turns a prologue chain into a closure raw-load -> value;
``build_reduction_epilogue_transform`` does the same on a scalar. Secondary tensor
operands are read from global memory at the in-scope (row, col) through their
strides, honouring the broadcast mode; comparisons become 1.0f / 0.0f.
"""

from __future__ import annotations

import math
import re
from typing import Callable

from metellus_b200.compute.elementwise import (
    BroadcastSpec,
    elementwise_arity,
    elementwise_expression,
    elementwise_outputs_bool,
)
from metellus_b200.orchestrator.assembly.extras import Extras, pname
from metellus_b200.orchestrator.ir import ElementwiseOp, Scalar, Tensor

ValueTransform = Callable[[str], str]

_IDENT = re.compile(r"\b(cond|x|y)\b")


def substitute(expr: str, **subs: str) -> str:
    """Replace the whole-word placeholders x / y / cond in an op template."""
    return _IDENT.sub(lambda m: subs.get(m.group(0), m.group(0)), expr)


def wrap_bool(op: str, expr: str) -> str:
    if elementwise_outputs_bool(op):
        return f"(({expr}) ? 1.0f : 0.0f)"
    return expr


def scalar_literal(value: float) -> str:
    """fp32 literal; exact for every float32 value (9 significant digits)."""
    if math.isnan(value):
        return "NAN"
    if math.isinf(value):
        return "INFINITY" if value > 0 else "(-INFINITY)"
    import numpy as np

    f = float(np.float32(value))
    if f == 0.0:
        return "-0.0f" if math.copysign(1.0, f) < 0 else "0.0f"
    return f"{f:.9e}f"


def operand_expr(operand: Tensor | Scalar, *, broadcast: BroadcastSpec, row_var: str, col_var: str) -> str:
    """Global read of one element of ``operand`` at the in-scope (row, col)."""
    if isinstance(operand, Scalar):
        return scalar_literal(operand.value)
    key = pname(operand.buffer_key)
    rs, cs = operand.row_stride, operand.col_stride

    def term(var: str, stride: int) -> str:
        return var if stride == 1 else f"(size_t){var} * {stride}ll"

    if len(operand.matrix_shape) == 1:
        # 1-D operand of a 1-D primary: indexed by the primary's row.
        return f"{key}[{term(row_var, rs)}]"
    if broadcast is BroadcastSpec.SCALAR:
        return f"{key}[0]"
    if broadcast is BroadcastSpec.ROW:
        return f"{key}[{term(col_var, cs)}]"
    if broadcast is BroadcastSpec.COL:
        return f"{key}[{term(row_var, rs)}]"
    return f"{key}[{term(row_var, rs)} + {term(col_var, cs)}]"


def chain_value_transform(
    chain: tuple[ElementwiseOp, ...],
    *,
    row_var: str,
    col_var: str,
    extras: Extras,
    base_slot: int,
) -> ValueTransform:
    """Prologue chain -> closure over the primary's raw load (expressions.py:117-170)."""
    if not chain:
        return lambda raw: raw
    primary = chain[0].operands[0]
    assert isinstance(primary, Tensor)
    available = {primary.name}
    for elem in chain:
        for operand in elem.operands[1:]:
            if isinstance(operand, Tensor) and operand.name not in available:
                extras.add_tensor(operand, base_slot)
        available.add(elem.out.name)

    def transform(raw: str) -> str:
        expr = raw
        values = {primary.name: raw}
        for elem in chain:
            tpl = elementwise_expression(elem.op)
            subs = {"x": f"({expr})"}
            modes = (elem.y_broadcast, elem.cond_broadcast)
            for k, key in ((1, "y"), (2, "cond")):
                if k < len(elem.operands):
                    o = elem.operands[k]
                    if isinstance(o, Tensor) and o.name in values:
                        subs[key] = f"({values[o.name]})"
                    else:
                        subs[key] = f"({operand_expr(o, broadcast=modes[k - 1], row_var=row_var, col_var=col_var)})"
            expr = wrap_bool(elem.op, substitute(tpl, **subs))
            values[elem.out.name] = expr
        return expr

    return transform


def build_reduction_epilogue_transform(chain: tuple[ElementwiseOp, ...]) -> ValueTransform:
    """Unary / Scalar-binary chain on the reduced scalar (expressions.py:173-205)."""
    steps: list[Callable[[str], str]] = []
    for elem in chain:
        tpl = elementwise_expression(elem.op)
        if elementwise_arity(elem.op) == 1:
            steps.append(lambda inner, t=tpl, n=elem.op: wrap_bool(n, substitute(t, x=f"({inner})")))
        else:
            y = elem.operands[1]
            assert isinstance(y, Scalar)
            lit = scalar_literal(y.value)
            steps.append(lambda inner, t=tpl, n=elem.op, lit=lit: wrap_bool(n, substitute(t, x=f"({inner})", y=f"({lit})")))

    def transform(v: str) -> str:
        for s in steps:
            v = s(v)
        return v

    return transform
