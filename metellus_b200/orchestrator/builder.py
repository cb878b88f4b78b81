"""``Operations``: the user-facing program builder (reference API:
src/orchestrator/builder.py:50-333).

A program is written against tensor *names*. The builder keeps one record per name
(its ``Tensor``: shape, strides, storage owner), the host arrays to upload, and the
ordered list of IR ops. Three kinds of call:

* declarations — ``input`` (shape only) and ``from_numpy`` (shape + payload);
* ops — ``matmul``, ``elementwise``, ``reduction`` and the copying ``reshape``;
  each creates exactly one new name (the IR is SSA), and the op's own constructor
  does the shape / broadcast / dtype validation;
* views — ``transpose`` and the metadata ``reshape``: a new name over the same
  storage, no op.

A failed op leaves the builder unchanged: the output name is registered only after
the op has been constructed. ``build()`` returns a copy of the op list, so the
builder can keep growing afterwards.

Batched (rank-3) tensors are accepted everywhere the IR accepts them; ``matmul``
infers ``a.shape[:-1] + (b.shape[-1],)`` as its output shape.
"""

from __future__ import annotations

import math
from typing import Callable

import numpy as np

from metellus_b200.compute.elementwise import BroadcastSpec
from metellus_b200.orchestrator.ir import (
    ElementwiseOp,
    Layout,
    MatmulOp,
    Op,
    OperandValue,
    Program,
    ReductionOp,
    Scalar,
    ShapeOp,
    Tensor,
)


def addressable_elements(t: Tensor) -> int:
    """How many elements of backing storage ``t`` can touch: one past the largest
    offset it addresses (``1`` for a scalar)."""
    strides = {0: (), 1: (t.row_stride,), 2: (t.row_stride, t.col_stride),
               3: (t.batch_stride, t.row_stride, t.col_stride)}[len(t.shape)]
    return 1 + sum((extent - 1) * stride for extent, stride in zip(t.shape, strides))


class Operations:
    """Builder for one program (mutable; ``build()`` snapshots the op list)."""

    def __init__(self, dtype: str = "float32") -> None:
        self._dtype = dtype
        self._by_name: dict[str, Tensor] = {}
        self._program: Program = []
        self._payloads: dict[str, np.ndarray] = {}

    # -- lookups --------------------------------------------------------------

    def _lookup(self, name: str) -> Tensor:
        try:
            return self._by_name[name]
        except KeyError:
            raise ValueError(f"tensor {name!r} is not declared: declare it with input() / from_numpy() "
                             "or produce it with an op first") from None

    def _require_fresh_view_name(self, out: str, what: str) -> None:
        if out in self._by_name:
            raise ValueError(f"{what} output {out!r} already declared; views need a new name")

    def _emit(self, out: str, shape: tuple[int, ...], make: Callable[[Tensor], Op]) -> Tensor:
        """Create op ``make(out_tensor)`` writing the new name ``out``; register the
        name and append the op only when construction (= validation) succeeded."""
        if out in self._by_name:
            raise ValueError(f"output tensor {out!r} already exists; the IR is SSA, so every op "
                             "needs a new output name")
        result = Tensor(name=out, shape=tuple(shape), dtype=self._dtype)
        op = make(result)
        self._by_name[out] = result
        self._program.append(op)
        return result

    # -- declarations ------------------------------------------------------------

    def input(self, name: str, shape: tuple[int, ...], layout: Layout = Layout.ROW_MAJOR,
              row_stride: int | None = None, col_stride: int | None = None) -> Tensor:
        """Declare a tensor the caller supplies (no producing op). Strides default to
        the contiguous ones for ``layout``. Re-declaring a name with the same shape
        returns the existing tensor; with another shape it is an error."""
        shape = tuple(shape)
        known = self._by_name.get(name)
        if known is not None:
            if known.shape != shape:
                raise ValueError(f"tensor {name!r} already declared with shape {known.shape}; "
                                 f"cannot declare it again as {shape}")
            return known
        t = Tensor(name=name, shape=shape, dtype=self._dtype, layout=layout,
                   row_stride=-1 if row_stride is None else row_stride,
                   col_stride=-1 if col_stride is None else col_stride)
        self._by_name[name] = t
        return t

    def from_numpy(self, arr: np.ndarray, name: str) -> Tensor:
        """Declare ``name`` with ``arr``'s shape and record ``arr`` as its upload.
        The array must be float32 (no silent widening or narrowing), ``name`` must
        own its storage (not a view), and the array must hold every element the
        tensor's strides can reach."""
        if arr.dtype != np.float32:
            raise ValueError(f"from_numpy({name!r}): the array must be float32, got {arr.dtype}")
        t = self.input(name, tuple(arr.shape))
        if t.buffer_key != name:
            raise ValueError(f"from_numpy: {name!r} is a view of {t.buffer_key!r}; only a storage owner "
                             "can receive an upload")
        if tuple(arr.shape) != t.shape:
            raise ValueError(f"from_numpy({name!r}): array shape {tuple(arr.shape)} differs from the "
                             f"declared shape {t.shape}")
        reach = addressable_elements(t)
        if arr.size < reach:
            raise ValueError(f"from_numpy({name!r}): the array has {arr.size} elements, but with "
                             f"row_stride={t.row_stride}, col_stride={t.col_stride} the tensor can address "
                             f"{reach} elements")
        self._payloads[name] = arr
        return t

    # -- ops -------------------------------------------------------------------

    def matmul(self, a: str, b: str, out: str) -> Tensor:
        """``out = a @ b`` (per batch index for rank-3 operands)."""
        ta, tb = self._lookup(a), self._lookup(b)
        return self._emit(out, ta.shape[:-1] + tb.shape[-1:], lambda o: MatmulOp(out=o, a=ta, b=tb))

    def elementwise(self, op: str, out: str, operands: tuple[str | int | float, ...],
                    y_broadcast: BroadcastSpec | str = BroadcastSpec.NONE,
                    cond_broadcast: BroadcastSpec | str = BroadcastSpec.NONE) -> Tensor:
        """Pointwise ``op``; the output has the first operand's shape. Operands are
        declared tensor names or Python numbers (inlined as ``Scalar`` constants);
        the first must be a tensor."""
        y_mode, cond_mode = BroadcastSpec(y_broadcast), BroadcastSpec(cond_broadcast)
        values: list[OperandValue] = [self._operand(o) for o in operands]
        if not values or not isinstance(values[0], Tensor):
            first = operands[0] if operands else None
            raise ValueError(f"elementwise {op!r}: operand[0] must be a tensor name, got {first!r}; "
                             "numbers may only be secondary operands")
        return self._emit(out, values[0].shape,
                          lambda o: ElementwiseOp(out=o, op=op, operands=tuple(values), y_broadcast=y_mode,
                                                  cond_broadcast=cond_mode))

    def _operand(self, o: str | int | float) -> OperandValue:
        if isinstance(o, str):
            return self._lookup(o)
        if isinstance(o, (int, float)) and not isinstance(o, bool):
            return Scalar(value=float(o))
        raise ValueError(f"operand {o!r} must be a tensor name (str) or a numeric literal (int / float)")

    def reduction(self, op: str, out: str, x: str, axis: int = -1) -> Tensor:
        """Reduce ``x`` along ``axis`` (the IR accepts the last axis only)."""
        from metellus_b200.compute.reduction import REDUCTION_OPS

        if op not in REDUCTION_OPS:
            raise ValueError(f"reduction op {op!r} is not one of {REDUCTION_OPS}")
        src = self._lookup(x)
        rank = len(src.shape)
        ax = axis + rank if axis < 0 else axis
        # the dropped axis, or (for an invalid axis) the last one, so that the IR op
        # reports the real problem
        keep = [d for i, d in enumerate(src.shape) if i != (ax if 0 <= ax < rank else rank - 1)]
        shape = tuple(keep) or (1,)
        return self._emit(out, shape, lambda o: ReductionOp(out=o, op=op, input=src, axis=axis))

    # -- views -----------------------------------------------------------------

    def transpose(self, name: str, out: str) -> Tensor:
        """``out`` = the transpose of ``name``'s (inner) matrix as a view: same storage,
        swapped shape and strides, no op."""
        src = self._lookup(name)
        self._require_fresh_view_name(out, "transpose")
        self._by_name[out] = view = src.transpose(out)
        return view

    def reshape(self, name: str, new_shape: tuple[int, ...], out: str) -> Tensor:
        """A metadata view when the source can be walked linearly (same storage, no
        op); otherwise a ``ShapeOp`` that gathers the source into a new contiguous
        1-D or 2-D tensor."""
        src = self._lookup(name)
        self._require_fresh_view_name(out, "reshape")
        target = tuple(new_shape)
        if src.can_reshape_as_view(target):
            self._by_name[out] = view = src.reshape_view(target, out)
            return view
        if not 1 <= len(target) <= 2:
            raise ValueError(f"a copying reshape needs a 1D or 2D target rank; got {target}")
        if math.prod(target) != src.element_count:
            raise ValueError(f"reshape element-count mismatch: {src.shape} has {src.element_count} elements, "
                             f"{target} has {math.prod(target)}")
        return self._emit(out, target, lambda o: ShapeOp(out=o, input=src))

    # -- results ---------------------------------------------------------------

    def build(self) -> Program:
        return list(self._program)

    @property
    def tensors(self) -> dict[str, Tensor]:
        return dict(self._by_name)

    @property
    def uploads(self) -> dict[str, np.ndarray]:
        return dict(self._payloads)
