"""The SSA IR the compiler works on (reference API: src/orchestrator/ir.py).

Four ops — matmul, elementwise, last-axis reduction, strided copy — each writing
one new tensor. A ``Tensor`` is a name, a shape and the strides at which its
elements sit in the storage of ``buffer_key`` (its own name, or the owner it is a
view of). Element ``(b, r, c)`` is at ``b * batch_stride + r * row_stride + c *
col_stride``; a 1-D tensor uses ``row_stride`` only and a scalar no stride.
Transposes and reshapes that only re-describe the same storage are views: new
tensors with the owner's ``buffer_key`` and different strides.

Every op checks its operand shapes, broadcast modes and dtypes when it is
constructed, and raises ``ValueError`` naming the problem; the builder relies on
that instead of checking twice.

Beyond the reference: rank-3 tensors ``(B, M, N)`` are batched matrices. Each op
then applies to every batch index independently (batched attention without B copies
of the program); broadcasts and reductions act on the inner matrix. Kernels map the
batch to ``gridDim.z`` and the multi-GPU runner shards it.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, replace
from enum import StrEnum

from metellus_b200.compute.elementwise import BroadcastSpec, elementwise_arity


class Layout(StrEnum):
    """Storage order of the (inner) matrix when no strides are given."""

    ROW_MAJOR = "row_major"
    COL_MAJOR = "col_major"


def _packed_strides(shape: tuple[int, ...], layout: Layout) -> tuple[int, int, int]:
    """(row_stride, col_stride, batch_stride) of a densely packed tensor: a matrix in
    ``layout`` order, batches back to back; a vector has step 1; a scalar none."""
    rank = len(shape)
    if rank > 3:
        raise ValueError(f"tensors have at most 3 dimensions (batch, rows, cols); got shape {shape}")
    if rank == 0:
        return 0, 0, 0
    if rank == 1:
        return 1, 0, 0
    rows, cols = shape[-2], shape[-1]
    rs, cs = (cols, 1) if layout is Layout.ROW_MAJOR else (1, rows)
    return rs, cs, (rows * cols if rank == 3 else 0)


@dataclass(frozen=True)
class Tensor:
    """An SSA value: ``name``, ``shape``, strides into ``buffer_key``'s storage.
    Strides left at -1 are filled in as the packed strides of ``layout``; an empty
    ``buffer_key`` means the tensor owns its storage."""

    name: str
    shape: tuple[int, ...]
    dtype: str = "float32"
    layout: Layout = Layout.ROW_MAJOR
    row_stride: int = -1
    col_stride: int = -1
    buffer_key: str = ""
    batch_stride: int = -1

    def __post_init__(self) -> None:
        if not all(d > 0 for d in self.shape):
            raise ValueError(f"every tensor dimension must be positive; got shape {self.shape}")
        packed = _packed_strides(tuple(self.shape), self.layout)
        for field, value in zip(("row_stride", "col_stride", "batch_stride"), packed):
            if getattr(self, field) == -1:
                object.__setattr__(self, field, value)
        if self.buffer_key == "":
            object.__setattr__(self, "buffer_key", self.name)

    # -- sizes ----------------------------------------------------------------

    @property
    def element_count(self) -> int:
        return math.prod(self.shape)

    @property
    def nbytes(self) -> int:
        return 4 * self.element_count   # the IR is fp32 throughout

    @property
    def batch(self) -> int:
        """The batch extent (1 below rank 3)."""
        return self.shape[0] if len(self.shape) == 3 else 1

    @property
    def matrix_shape(self) -> tuple[int, ...]:
        """The shape of one batch entry (the shape itself below rank 3)."""
        return tuple(self.shape[-2:]) if len(self.shape) == 3 else tuple(self.shape)

    def _dims(self) -> list[tuple[int, int]]:
        """(extent, stride) per dimension, outermost first."""
        strides = {1: (self.row_stride,), 2: (self.row_stride, self.col_stride),
                   3: (self.batch_stride, self.row_stride, self.col_stride)}.get(len(self.shape), ())
        return list(zip(self.shape, strides))

    # -- views ----------------------------------------------------------------

    def linear_step(self) -> int | None:
        """The step ``s`` such that visiting the elements in row-major order reads
        storage offsets 0, s, 2s, ... — or None when no single step does. Dimensions
        of extent 1 never break linearity; with every extent 1 the step is the
        innermost dimension's stride (1 for a scalar)."""
        dims = self._dims()
        if not dims:
            return 1
        live = [(n, s) for n, s in dims if n > 1]
        if not live:
            return dims[-1][1]
        step = live[-1][1]
        span = step
        for n, s in reversed(live):
            if s != span:
                return None
            span = n * s
        return step

    def is_contiguous(self) -> bool:
        return self.linear_step() == 1

    def transpose(self, name: str) -> Tensor:
        """A view of the transposed (inner) matrix: shape and strides of the last two
        dimensions swapped, the layout flipped, nothing copied."""
        if len(self.shape) not in (2, 3):
            raise ValueError(f"transpose is 2D-only (a matrix or a batch of matrices); got shape {self.shape}")
        flipped = Layout.COL_MAJOR if self.layout is Layout.ROW_MAJOR else Layout.ROW_MAJOR
        return replace(self, name=name, shape=self.shape[:-2] + (self.shape[-1], self.shape[-2]), layout=flipped,
                       row_stride=self.col_stride, col_stride=self.row_stride)

    def can_reshape_as_view(self, new_shape: tuple[int, ...]) -> bool:
        """A reshape can alias the storage when the shape is unchanged, or when the
        new shape (rank 1-3) has the same element count and this tensor can be walked
        with one linear step."""
        target = tuple(new_shape)
        if target == self.shape:
            return True
        return (1 <= len(target) <= 3 and math.prod(target) == self.element_count
                and self.linear_step() is not None)

    def reshape_view(self, new_shape: tuple[int, ...], name: str) -> Tensor:
        """The view ``can_reshape_as_view`` allows: the same strides for an unchanged
        shape, else row-major strides scaled by the linear step."""
        target = tuple(new_shape)
        if not self.can_reshape_as_view(target):
            raise ValueError(f"cannot reshape {self.name!r} {self.shape} -> {target} as a view: that needs the "
                             "same shape, or a linearly-iterable source with the same element count")
        if target == self.shape:
            return replace(self, name=name)
        step = self.linear_step()
        packed = _packed_strides(target, Layout.ROW_MAJOR)
        rs, cs, bs = (p * step for p in packed)
        return Tensor(name=name, shape=target, dtype=self.dtype, layout=Layout.ROW_MAJOR, row_stride=rs,
                      col_stride=cs, buffer_key=self.buffer_key, batch_stride=bs)


@dataclass(frozen=True)
class Scalar:
    """A constant elementwise operand, inlined into the kernel as a literal."""

    value: float


OperandValue = Tensor | Scalar


def _broadcast_shape(primary: tuple[int, ...], mode: BroadcastSpec) -> tuple[int, ...]:
    """The shape a secondary operand must have under ``mode`` against a primary of
    shape ``primary``: the same shape (NONE), 1 x 1 (SCALAR), 1 x N (ROW) or M x 1
    (COL); a batched primary keeps its batch extent."""
    if mode is BroadcastSpec.NONE:
        return primary
    if len(primary) not in (2, 3):
        raise ValueError(f"broadcast={mode!r} needs a 2D (or batched 2D) primary; got shape {primary}")
    *batch, m, n = primary
    inner = {BroadcastSpec.SCALAR: (1, 1), BroadcastSpec.ROW: (1, n), BroadcastSpec.COL: (m, 1)}[mode]
    return tuple(batch) + inner


def _check_secondary(role: str, primary: Tensor, operand: OperandValue, mode: BroadcastSpec) -> None:
    if isinstance(operand, Scalar):
        if mode is not BroadcastSpec.NONE:
            raise ValueError(f"{role}_broadcast={mode!r} cannot be set for a Scalar operand: scalars are inlined "
                             "as literals, not broadcast")
        return
    want = _broadcast_shape(primary.shape, mode)
    if operand.shape == want:
        return
    if mode is BroadcastSpec.NONE:
        raise ValueError(f"{role}-operand shape {operand.shape} must match primary {primary.shape} when "
                         f"{role}_broadcast=NONE")
    raise ValueError(f"{role}-operand shape {operand.shape} incompatible with {role}_broadcast={mode!r} "
                     f"(expected {want})")


@dataclass(frozen=True)
class MatmulOp:
    """``out = a @ b``; for rank-3 operands, per batch index."""

    out: Tensor
    a: Tensor
    b: Tensor

    def __post_init__(self) -> None:
        a, b = self.a.shape, self.b.shape
        if len(a) != len(b) or len(a) not in (2, 3):
            raise ValueError(f"matmul operands must both be 2D (or both batched 3D); got a={a}, b={b}")
        if len(a) == 3 and a[0] != b[0]:
            raise ValueError(f"matmul batch mismatch: a={a}, b={b}")
        if a[-1] != b[-2]:
            raise ValueError(f"matmul contraction-axis mismatch: a={a} has {a[-1]} columns, b={b} has {b[-2]} rows")
        if self.out.shape != a[:-1] + b[-1:]:
            raise ValueError(f"matmul out shape {self.out.shape} does not match a @ b = {a[:-1] + b[-1:]}")
        if len({self.a.dtype, self.b.dtype, self.out.dtype}) != 1:
            raise ValueError(f"matmul dtypes must match; got a={self.a.dtype}, b={self.b.dtype}, "
                             f"out={self.out.dtype}")

    @property
    def inputs(self) -> tuple[Tensor, ...]:
        return (self.a, self.b)


@dataclass(frozen=True)
class ElementwiseOp:
    """A pointwise op from the elementwise expression table, on 1-3 operands. The
    first operand is a tensor of the output's shape; a second (``y``) and third
    (``cond``) operand are tensors broadcast by ``y_broadcast`` / ``cond_broadcast``,
    or scalars."""

    out: Tensor
    op: str
    operands: tuple[OperandValue, ...]
    y_broadcast: BroadcastSpec = BroadcastSpec.NONE
    cond_broadcast: BroadcastSpec = BroadcastSpec.NONE

    def __post_init__(self) -> None:
        arity = elementwise_arity(self.op)
        if len(self.operands) != arity:
            raise ValueError(f"elementwise {self.op!r} is arity-{arity}, got {len(self.operands)} operands")
        primary = self.operands[0]
        if not isinstance(primary, Tensor):
            raise ValueError(f"elementwise {self.op!r}: operand[0] must be a tensor, got {primary!r}; scalars "
                             "may only be secondary operands")
        if self.out.shape != primary.shape:
            raise ValueError(f"elementwise out shape {self.out.shape} must match primary operand shape "
                             f"{primary.shape}")
        for position, role, mode in ((1, "y", self.y_broadcast), (2, "cond", self.cond_broadcast)):
            if position < arity:
                _check_secondary(role, primary, self.operands[position], mode)
            elif mode is not BroadcastSpec.NONE:
                raise ValueError(f"{role}_broadcast={mode!r} set on arity-{arity} op {self.op!r}")

    @property
    def inputs(self) -> tuple[Tensor, ...]:
        return tuple(o for o in self.operands if isinstance(o, Tensor))


@dataclass(frozen=True)
class ReductionOp:
    """Reduce the last axis: (M, K) -> (M,), batched (B, M, K) -> (B, M)."""

    out: Tensor
    op: str
    input: Tensor
    axis: int = -1

    def __post_init__(self) -> None:
        shape = self.input.shape
        if len(shape) not in (2, 3):
            raise ValueError(f"reduction input must be 2D (or batched 3D); got shape {shape}")
        if self.axis not in (len(shape) - 1, -1):
            raise ValueError(f"reduction supports the last axis only; got axis={self.axis} on shape {shape}")
        if self.out.shape != shape[:-1]:
            raise ValueError(f"reduction out shape {self.out.shape} does not match input {shape} reduced along "
                             f"axis {self.axis} (expected {shape[:-1]})")

    @property
    def inputs(self) -> tuple[Tensor, ...]:
        return (self.input,)


@dataclass(frozen=True)
class ShapeOp:
    """Copy ``input`` (read through its strides, in logical row-major order) into
    ``out``, a new packed tensor with the same element count."""

    out: Tensor
    input: Tensor

    def __post_init__(self) -> None:
        src, dst = self.input, self.out
        if src.element_count != dst.element_count:
            raise ValueError(f"shape op element-count mismatch: input {src.shape} ({src.element_count} elements) "
                             f"-> out {dst.shape} ({dst.element_count} elements)")
        if src.dtype != dst.dtype:
            raise ValueError(f"shape op dtype mismatch: input {src.dtype!r} -> out {dst.dtype!r}")
        if dst.buffer_key != dst.name:
            raise ValueError(f"shape op out must own its storage (buffer_key == name); got name={dst.name!r}, "
                             f"buffer_key={dst.buffer_key!r}")

    @property
    def inputs(self) -> tuple[Tensor, ...]:
        return (self.input,)


Op = MatmulOp | ElementwiseOp | ReductionOp | ShapeOp
Program = list[Op]
