"""Strided-copy strategy for ShapeOp (reference: assembly/shape.py:14-68): one
grid-stride pass reading the source through its strides, writing the output
contiguously."""

from __future__ import annotations

from metellus_b200.compute.copy import StridedCopyFragment
from metellus_b200.compute.fragments import CodegenContext
from metellus_b200.orchestrator.assembly.decision import DecisionView
from metellus_b200.orchestrator.assembly.extras import param_decl, pname
from metellus_b200.orchestrator.ir import ShapeOp
from metellus_b200.orchestrator.kernel_group import KernelGroup
from metellus_b200.runtime.program import Kernel


def assemble_shape(decision: DecisionView, function_name: str | None) -> KernelGroup:
    op = decision.shape_op
    assert isinstance(op, ShapeOp)
    src, out = op.input, op.out
    n = out.element_count
    if len(src.shape) == 3:
        raise ValueError("ShapeOp of a batched tensor is not supported; reshape per batch instead")
    if len(src.shape) == 2:
        cols, rs, cs = src.shape[1], src.row_stride, src.col_stride
    else:
        cols, rs, cs = src.shape[0], 0, src.row_stride
    nt = 256
    grid_x = max(1, min((n + nt - 1) // nt, 148 * 8))
    frag = StridedCopyFragment(input_name=pname(src.buffer_key), output_name=pname(out.buffer_key),
                               input_row_stride=rs, input_col_stride=cs, input_cols=cols)
    fn = function_name or f"shape_{out.name}"
    ctx = CodegenContext(function_name=fn, buffers=(param_decl(src.buffer_key), param_decl(out.buffer_key, writable=True)),
                         dims=("N",), tg_x=nt, tg_y=1)
    return KernelGroup(kernel=Kernel(fragments=(frag,), ctx=ctx), bindings=(src.buffer_key, out.buffer_key),
                       dims=(n,), grid=(grid_x, 1, 1), threads=(nt, 1, 1), ops=(op,), strategy=decision.strategy)
