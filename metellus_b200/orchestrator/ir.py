"""Lowered-primitive SSA IR: matmul, elementwise, last-axis reduction, strided copy.

Behaviour follows the reference IR (src/orchestrator/ir.py): every op defines one
fresh output tensor, shapes and broadcast modes are validated in ``__post_init__``,
and views (transpose / metadata reshape) alias the storage owner through
``buffer_key`` (ir.py:54-96).

One extension over the reference: tensors may carry a leading *batch* dimension,
``shape == (B, M, N)``. Every op then applies independently per batch index, which is
how batched attention (B independent S x S problems) is expressed without unrolling
the program B times. Rank <= 2 behaviour is unchanged. The batch dimension maps to
``gridDim.z`` in the generated kernels and is the unit the multi-GPU runner shards.
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import StrEnum

from metellus_b200.compute.elementwise import BroadcastSpec, elementwise_arity


class Layout(StrEnum):
    """Logical storage order of the inner 2-D matrix (ir.py:27-33)."""

    ROW_MAJOR = "row_major"
    COL_MAJOR = "col_major"


def _default_strides(shape: tuple[int, ...], layout: Layout) -> tuple[int, int, int]:
    """Contiguous (row_stride, col_stride, batch_stride) in elements.

    1-D: (1, 0, 0); 0-D: (0, 0, 0) as in the reference (ir.py:36-50). For rank 3 the
    inner (M, N) matrix follows ``layout`` and batches are packed back to back."""
    if len(shape) == 0:
        return (0, 0, 0)
    if len(shape) == 1:
        return (1, 0, 0)
    if len(shape) == 2:
        M, N = shape
        return (N, 1, 0) if layout is Layout.ROW_MAJOR else (1, M, 0)
    if len(shape) == 3:
        _, M, N = shape
        rs, cs = (N, 1) if layout is Layout.ROW_MAJOR else (1, M)
        return (rs, cs, M * N)
    raise ValueError(f"tensors are 0D..3D (batch, rows, cols); got shape {shape}")


@dataclass(frozen=True)
class Tensor:
    """An SSA value; ``buffer_key`` names the storage owner (ir.py:53-96).

    Element (b, r, c) lives at ``b*batch_stride + r*row_stride + c*col_stride``.
    For rank <= 2 ``batch_stride`` is 0 and the formula reduces to the reference's."""

    name: str
    shape: tuple[int, ...]
    dtype: str = "float32"
    layout: Layout = Layout.ROW_MAJOR
    row_stride: int = -1
    col_stride: int = -1
    buffer_key: str = ""
    batch_stride: int = -1

    def __post_init__(self) -> None:
        if any(d <= 0 for d in self.shape):
            raise ValueError(f"tensor dimensions must be positive; got shape {self.shape}")
        rs, cs, bs = _default_strides(tuple(self.shape), self.layout)
        if self.row_stride == -1:
            object.__setattr__(self, "row_stride", rs)
        if self.col_stride == -1:
            object.__setattr__(self, "col_stride", cs)
        if self.batch_stride == -1:
            object.__setattr__(self, "batch_stride", bs)
        if not self.buffer_key:
            object.__setattr__(self, "buffer_key", self.name)

    # -- sizes --------------------------------------------------------------

    @property
    def nbytes(self) -> int:
        return 4 * self.element_count  # fp32 only, as in the reference (ir.py:98-103)

    @property
    def element_count(self) -> int:
        n = 1
        for d in self.shape:
            n *= d
        return n

    @property
    def batch(self) -> int:
        """Leading batch extent (1 for rank <= 2)."""
        return self.shape[0] if len(self.shape) == 3 else 1

    @property
    def matrix_shape(self) -> tuple[int, ...]:
        """The per-batch shape (drops the batch dim of a rank-3 tensor)."""
        return tuple(self.shape[1:]) if len(self.shape) == 3 else tuple(self.shape)

    # -- views ----------------------------------------------------------------

    def linear_step(self) -> int | None:
        """Step ``c`` such that row-major iteration visits offsets 0, c, 2c, ...;
        None when iteration is non-linear (ir.py:112-146, extended to rank 3)."""
        if len(self.shape) == 0:
            return 1
        if len(self.shape) == 1:
            return self.row_stride
        if len(self.shape) == 2:
            M, K = self.shape
            if M == 1:
                return self.col_stride
            if K == 1:
                return self.row_stride
            if self.row_stride == K * self.col_stride:
                return self.col_stride
            return None
        B, M, K = self.shape
        inner = Tensor("_", (M, K), row_stride=self.row_stride, col_stride=self.col_stride)
        c = inner.linear_step()
        if c is None:
            return None
        if B == 1:
            return c
        if M * K == 1:
            return self.batch_stride
        if self.batch_stride == M * K * c:
            return c
        return None

    def is_contiguous(self) -> bool:
        return self.linear_step() == 1

    def transpose(self, name: str) -> Tensor:
        """Logical transpose of the inner matrix, no data movement (ir.py:154-174)."""
        if len(self.shape) not in (2, 3):
            raise ValueError(f"transpose is 2D-only (a 2D or batched 2D tensor); got shape {self.shape}")
        new_layout = Layout.COL_MAJOR if self.layout is Layout.ROW_MAJOR else Layout.ROW_MAJOR
        if len(self.shape) == 2:
            M, N = self.shape
            new_shape: tuple[int, ...] = (N, M)
        else:
            B, M, N = self.shape
            new_shape = (B, N, M)
        return Tensor(
            name=name,
            shape=new_shape,
            dtype=self.dtype,
            layout=new_layout,
            row_stride=self.col_stride,
            col_stride=self.row_stride,
            buffer_key=self.buffer_key,
            batch_stride=self.batch_stride,
        )

    def can_reshape_as_view(self, new_shape: tuple[int, ...]) -> bool:
        """Same shape, or same element count + linear source (ir.py:176-200)."""
        new_shape_t = tuple(new_shape)
        if new_shape_t == self.shape:
            return True
        if len(new_shape_t) > 3 or len(new_shape_t) == 0:
            return False
        prod = 1
        for d in new_shape_t:
            prod *= d
        if prod != self.element_count:
            return False
        return self.linear_step() is not None

    def reshape_view(self, new_shape: tuple[int, ...], name: str) -> Tensor:
        """Metadata reshape aliasing this buffer (ir.py:202-246)."""
        if not self.can_reshape_as_view(new_shape):
            raise ValueError(
                f"cannot reshape {self.name!r} {self.shape} -> {tuple(new_shape)} "
                "as a metadata swap: needs same shape OR a linearly-iterable "
                "source with matching element count"
            )
        new_shape_t = tuple(new_shape)
        if new_shape_t == self.shape:
            return Tensor(
                name=name,
                shape=self.shape,
                dtype=self.dtype,
                layout=self.layout,
                row_stride=self.row_stride,
                col_stride=self.col_stride,
                buffer_key=self.buffer_key,
                batch_stride=self.batch_stride,
            )
        c = self.linear_step()
        assert c is not None
        if len(new_shape_t) == 1:
            rs, cs, bs = c, 0, 0
        elif len(new_shape_t) == 2:
            rs, cs, bs = new_shape_t[1] * c, c, 0
        else:
            _, M2, N2 = new_shape_t
            rs, cs, bs = N2 * c, c, M2 * N2 * c
        return Tensor(
            name=name,
            shape=new_shape_t,
            dtype=self.dtype,
            layout=Layout.ROW_MAJOR,
            row_stride=rs,
            col_stride=cs,
            buffer_key=self.buffer_key,
            batch_stride=bs,
        )


@dataclass(frozen=True)
class Scalar:
    """Compile-time constant elementwise operand, inlined as a literal (ir.py:249-256)."""

    value: float


OperandValue = Tensor | Scalar


def _expected_broadcast_shape(
    primary_shape: tuple[int, ...], mode: BroadcastSpec
) -> tuple[int, ...]:
    """Operand shape implied by ``mode`` (ir.py:262-278). For a batched primary the
    broadcast applies to the inner matrix and the batch dim is kept."""
    if mode is BroadcastSpec.NONE:
        return primary_shape
    if len(primary_shape) not in (2, 3):
        raise ValueError(f"broadcast={mode!r} requires a 2D primary; got shape {primary_shape}")
    if len(primary_shape) == 2:
        M, N = primary_shape
        lead: tuple[int, ...] = ()
    else:
        B, M, N = primary_shape
        lead = (B,)
    return lead + {
        BroadcastSpec.SCALAR: (1, 1),
        BroadcastSpec.ROW: (1, N),
        BroadcastSpec.COL: (M, 1),
    }[mode]


def _check_operand_broadcast(
    label: str, primary: Tensor, operand: OperandValue, mode: BroadcastSpec
) -> None:
    """Validate one secondary operand (ir.py:281-308)."""
    if isinstance(operand, Scalar):
        if mode is not BroadcastSpec.NONE:
            raise ValueError(
                f"{label}_broadcast={mode!r} cannot be set for a Scalar "
                "operand — scalars are inlined, not broadcast"
            )
        return
    expected = _expected_broadcast_shape(primary.shape, mode)
    if operand.shape != expected:
        if mode is BroadcastSpec.NONE:
            raise ValueError(
                f"{label}-operand shape {operand.shape} must match "
                f"primary {primary.shape} when {label}_broadcast=NONE"
            )
        raise ValueError(
            f"{label}-operand shape {operand.shape} incompatible "
            f"with {label}_broadcast={mode!r} (expected {expected})"
        )


@dataclass(frozen=True)
class MatmulOp:
    """out = a @ b (ir.py:311-348); batched operands multiply per batch index."""

    out: Tensor
    a: Tensor
    b: Tensor

    def __post_init__(self) -> None:
        ra, rb = len(self.a.shape), len(self.b.shape)
        if ra != rb or ra not in (2, 3):
            raise ValueError(
                f"matmul operands must be 2D (or both batched 3D); got a={self.a.shape}, b={self.b.shape}"
            )
        if ra == 3 and self.a.shape[0] != self.b.shape[0]:
            raise ValueError(f"matmul batch mismatch: a={self.a.shape}, b={self.b.shape}")
        if self.a.shape[-1] != self.b.shape[-2]:
            raise ValueError(f"matmul contraction-axis mismatch: a={self.a.shape}, b={self.b.shape}")
        expected = self.a.shape[:-1] + (self.b.shape[-1],)
        if self.out.shape != expected:
            raise ValueError(f"matmul out shape {self.out.shape} does not match a @ b = {expected}")
        if not (self.a.dtype == self.b.dtype == self.out.dtype):
            raise ValueError(
                f"matmul dtypes must match; got a={self.a.dtype}, "
                f"b={self.b.dtype}, out={self.out.dtype}"
            )

    @property
    def inputs(self) -> tuple[Tensor, ...]:
        return (self.a, self.b)


@dataclass(frozen=True)
class ElementwiseOp:
    """Pointwise op over the names in ``UNARY/BINARY/TERNARY_EXPRESSIONS``
    (ir.py:351-413)."""

    out: Tensor
    op: str
    operands: tuple[OperandValue, ...]
    y_broadcast: BroadcastSpec = BroadcastSpec.NONE
    cond_broadcast: BroadcastSpec = BroadcastSpec.NONE

    def __post_init__(self) -> None:
        arity = elementwise_arity(self.op)
        if len(self.operands) != arity:
            raise ValueError(
                f"elementwise {self.op!r} is arity-{arity}, got {len(self.operands)} operands"
            )
        primary = self.operands[0]
        if not isinstance(primary, Tensor):
            raise ValueError(
                f"elementwise {self.op!r}: operand[0] must be a Tensor; "
                f"got {primary!r}. Scalars are only allowed as secondary operands."
            )
        if self.out.shape != primary.shape:
            raise ValueError(
                f"elementwise out shape {self.out.shape} must match "
                f"primary operand shape {primary.shape}"
            )
        if arity >= 2:
            _check_operand_broadcast("y", primary, self.operands[1], self.y_broadcast)
        elif self.y_broadcast is not BroadcastSpec.NONE:
            raise ValueError(f"y_broadcast={self.y_broadcast!r} set on arity-1 op {self.op!r}")
        if arity == 3:
            _check_operand_broadcast("cond", primary, self.operands[2], self.cond_broadcast)
        elif self.cond_broadcast is not BroadcastSpec.NONE:
            raise ValueError(
                f"cond_broadcast={self.cond_broadcast!r} set on arity-{arity} op {self.op!r}"
            )

    @property
    def inputs(self) -> tuple[Tensor, ...]:
        return tuple(o for o in self.operands if isinstance(o, Tensor))


@dataclass(frozen=True)
class ReductionOp:
    """Last-axis reduction (ir.py:416-449); a batched (B, M, K) input reduces to
    (B, M)."""

    out: Tensor
    op: str
    input: Tensor
    axis: int = -1

    def __post_init__(self) -> None:
        rank = len(self.input.shape)
        if rank not in (2, 3):
            raise ValueError(f"reduction input must be 2D (or batched 3D); got shape {self.input.shape}")
        normalized = self.axis if self.axis >= 0 else rank + self.axis
        if normalized != rank - 1:
            raise ValueError(
                f"reduction supports last axis only; got axis={self.axis} on shape {self.input.shape}"
            )
        expected = self.input.shape[:normalized] + self.input.shape[normalized + 1 :]
        if self.out.shape != expected:
            raise ValueError(
                f"reduction out shape {self.out.shape} does not match "
                f"input {self.input.shape} reduced along axis {self.axis} "
                f"(expected {expected})"
            )

    @property
    def inputs(self) -> tuple[Tensor, ...]:
        return (self.input,)


@dataclass(frozen=True)
class ShapeOp:
    """Strided gather into a fresh contiguous buffer (ir.py:452-487)."""

    out: Tensor
    input: Tensor

    def __post_init__(self) -> None:
        if self.input.element_count != self.out.element_count:
            raise ValueError(
                f"shape op element-count mismatch: input {self.input.shape} "
                f"({self.input.element_count} elems) -> out {self.out.shape} "
                f"({self.out.element_count} elems)"
            )
        if self.input.dtype != self.out.dtype:
            raise ValueError(
                f"shape op dtype mismatch: input {self.input.dtype!r} -> out {self.out.dtype!r}"
            )
        if self.out.buffer_key != self.out.name:
            raise ValueError(
                "shape op out must own its buffer (buffer_key == name); "
                f"got name={self.out.name!r}, buffer_key={self.out.buffer_key!r}"
            )

    @property
    def inputs(self) -> tuple[Tensor, ...]:
        return (self.input,)


Op = MatmulOp | ElementwiseOp | ReductionOp | ShapeOp
Program = list[Op]
