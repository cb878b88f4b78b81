"""``Operations``: the name-resolution builder for the IR (builder.py:50-333).

Callers name tensors by string; the builder keeps a name -> Tensor registry, records
numpy uploads, and appends validated ops. Views (transpose / metadata reshape) are
registry entries, not ops; a reshape that cannot be a view becomes a ``ShapeOp``.
"""

from __future__ import annotations

import numpy as np

from metellus_b200.compute.elementwise import BroadcastSpec
from metellus_b200.orchestrator.ir import (
    ElementwiseOp,
    Layout,
    MatmulOp,
    OperandValue,
    Program,
    ReductionOp,
    Scalar,
    ShapeOp,
    Tensor,
)


class Operations:
    """Mutable program builder. ``build()`` returns a fresh op-list snapshot."""

    def __init__(self, dtype: str = "float32") -> None:
        self._dtype = dtype
        self._tensors: dict[str, Tensor] = {}
        self._ops: Program = []
        self._uploads: dict[str, np.ndarray] = {}

    # -- tensor registry -----------------------------------------------------

    def input(
        self,
        name: str,
        shape: tuple[int, ...],
        layout: Layout = Layout.ROW_MAJOR,
        row_stride: int | None = None,
        col_stride: int | None = None,
    ) -> Tensor:
        """Declare a caller-supplied tensor (builder.py:62-79)."""
        return self._declare(name, shape, layout=layout, row_stride=row_stride,
                             col_stride=col_stride)

    def from_numpy(self, arr: np.ndarray, name: str) -> Tensor:
        """Declare an input and record its payload (builder.py:81-114). Only float32
        storage owners are accepted."""
        if arr.dtype != np.float32:
            raise ValueError(f"from_numpy: array dtype must be float32; got {arr.dtype}")
        t = self._declare(name, tuple(arr.shape))
        if t.buffer_key != name:
            raise ValueError(
                f"from_numpy: {name!r} is a view of {t.buffer_key!r}; only "
                "storage owners can be uploaded"
            )
        if tuple(arr.shape) != t.shape:
            raise ValueError(
                f"from_numpy: array shape {tuple(arr.shape)} does not match "
                f"declared tensor shape {t.shape}"
            )
        required = _required_storage_elements(t)
        if arr.size < required:
            raise ValueError(
                f"from_numpy: array with shape {tuple(arr.shape)} provides {arr.size} "
                f"elements, but tensor {name!r} with strides (row_stride={t.row_stride}, "
                f"col_stride={t.col_stride}) can address {required} elements"
            )
        self._uploads[name] = arr
        return t

    def _declare(
        self,
        name: str,
        shape: tuple[int, ...],
        *,
        layout: Layout = Layout.ROW_MAJOR,
        row_stride: int | None = None,
        col_stride: int | None = None,
    ) -> Tensor:
        existing = self._tensors.get(name)
        if existing is not None:
            if existing.shape != tuple(shape):
                raise ValueError(
                    f"tensor {name!r} already declared with shape {existing.shape}, "
                    f"cannot redeclare as {tuple(shape)}"
                )
            return existing
        t = Tensor(
            name=name,
            shape=tuple(shape),
            dtype=self._dtype,
            layout=layout,
            row_stride=-1 if row_stride is None else row_stride,
            col_stride=-1 if col_stride is None else col_stride,
        )
        self._tensors[name] = t
        return t

    def _bind_existing(self, name: str) -> Tensor:
        t = self._tensors.get(name)
        if t is None:
            raise ValueError(
                f"tensor {name!r} is not declared — call ops.input(...) first "
                "or use an op that produces it"
            )
        return t

    def _reserve_output(self, name: str, shape: tuple[int, ...]) -> Tensor:
        if name in self._tensors:
            raise ValueError(f"output tensor {name!r} already defined; IR is SSA — pick a fresh name")
        return Tensor(name=name, shape=tuple(shape), dtype=self._dtype)

    def _commit_output(self, t: Tensor) -> None:
        self._tensors[t.name] = t

    # -- ops -------------------------------------------------------------------

    def matmul(self, a: str, b: str, out: str) -> Tensor:
        a_t = self._bind_existing(a)
        b_t = self._bind_existing(b)
        out_t = self._reserve_output(out, a_t.shape[:-1] + (b_t.shape[-1],))
        op = MatmulOp(out=out_t, a=a_t, b=b_t)
        self._commit_output(out_t)
        self._ops.append(op)
        return out_t

    def elementwise(
        self,
        op: str,
        out: str,
        operands: tuple[str | int | float, ...],
        y_broadcast: BroadcastSpec | str = BroadcastSpec.NONE,
        cond_broadcast: BroadcastSpec | str = BroadcastSpec.NONE,
    ) -> Tensor:
        """Pointwise op; numeric literals become ``Scalar`` operands (builder.py:183-235)."""
        y_bc = BroadcastSpec(y_broadcast)
        cond_bc = BroadcastSpec(cond_broadcast)
        resolved: list[OperandValue] = []
        for o in operands:
            if isinstance(o, str):
                resolved.append(self._bind_existing(o))
            elif isinstance(o, (int, float)) and not isinstance(o, bool):
                resolved.append(Scalar(value=float(o)))
            else:
                raise ValueError(
                    f"operand {o!r} must be a tensor name (str) or numeric literal (int/float)"
                )
        primary = resolved[0] if resolved else None
        if not isinstance(primary, Tensor):
            raise ValueError(
                f"elementwise {op!r}: operand[0] must be a tensor name; got "
                f"{operands[0] if operands else None!r}. Scalars are only allowed as "
                "secondary operands."
            )
        out_t = self._reserve_output(out, primary.shape)
        ew = ElementwiseOp(out=out_t, op=op, operands=tuple(resolved), y_broadcast=y_bc,
                           cond_broadcast=cond_bc)
        self._commit_output(out_t)
        self._ops.append(ew)
        return out_t

    def transpose(self, name: str, out: str) -> Tensor:
        """Logical transpose view; no op is emitted (builder.py:237-249)."""
        src = self._bind_existing(name)
        if out in self._tensors:
            raise ValueError(f"view tensor {out!r} already declared; pick a fresh name")
        view = src.transpose(out)
        self._tensors[out] = view
        return view

    def reshape(self, name: str, new_shape: tuple[int, ...], out: str) -> Tensor:
        """Metadata view when possible, ``ShapeOp`` copy otherwise (builder.py:251-294)."""
        src = self._bind_existing(name)
        if out in self._tensors:
            raise ValueError(f"reshape output {out!r} already declared; pick a fresh name")
        new_shape_t = tuple(new_shape)
        if src.can_reshape_as_view(new_shape_t):
            view = src.reshape_view(new_shape_t, out)
            self._tensors[out] = view
            return view
        if len(new_shape_t) == 0 or len(new_shape_t) > 2:
            raise ValueError(f"reshape target rank must be 1D or 2D; got {new_shape_t}")
        prod = 1
        for d in new_shape_t:
            prod *= d
        if prod != src.element_count:
            raise ValueError(
                f"reshape element-count mismatch: {src.shape} ({src.element_count}) -> "
                f"{new_shape_t} ({prod})"
            )
        out_t = self._reserve_output(out, new_shape_t)
        op = ShapeOp(out=out_t, input=src)
        self._commit_output(out_t)
        self._ops.append(op)
        return out_t

    def reduction(self, op: str, out: str, x: str, axis: int = -1) -> Tensor:
        """Last-axis reduction (builder.py:296-317)."""
        from metellus_b200.compute.reduction import REDUCTION_OPS

        if op not in REDUCTION_OPS:
            raise ValueError(f"reduction op {op!r} not in {REDUCTION_OPS}")
        x_t = self._bind_existing(x)
        normalized = axis if axis >= 0 else len(x_t.shape) + axis
        if 0 <= normalized < len(x_t.shape):
            out_shape = x_t.shape[:normalized] + x_t.shape[normalized + 1 :]
        else:
            out_shape = x_t.shape[:-1] or (1,)
        out_t = self._reserve_output(out, out_shape)
        red = ReductionOp(out=out_t, op=op, input=x_t, axis=axis)
        self._commit_output(out_t)
        self._ops.append(red)
        return out_t

    # -- finalize ----------------------------------------------------------------

    def build(self) -> Program:
        return list(self._ops)

    @property
    def tensors(self) -> dict[str, Tensor]:
        return dict(self._tensors)

    @property
    def uploads(self) -> dict[str, np.ndarray]:
        return dict(self._uploads)


def _required_storage_elements(t: Tensor) -> int:
    if len(t.shape) == 0:
        return 1
    if len(t.shape) == 1:
        return (t.shape[0] - 1) * t.row_stride + 1
    if len(t.shape) == 2:
        rows, cols = t.shape
        return (rows - 1) * t.row_stride + (cols - 1) * t.col_stride + 1
    b, rows, cols = t.shape
    return (b - 1) * t.batch_stride + (rows - 1) * t.row_stride + (cols - 1) * t.col_stride + 1
