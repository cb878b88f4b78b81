"""Reduction strategies: standalone, prologue-fused, epilogue-fused last-axis
reduction (reference template: assembly/reduction.py:24-109). One 256-thread block
per row; slots: input 0, output 1, chain extras after."""

from __future__ import annotations

from metellus_b200.compute.fragments import CodegenContext
from metellus_b200.compute.reduction import (
    COLRED_COLS,
    COLRED_WARPS,
    ColumnReductionFragment,
    LastAxisReductionComputeFragment,
    LastAxisReductionSetupFragment,
    StoreReductionResultFragment,
)
from metellus_b200.orchestrator.assembly.decision import DecisionView
from metellus_b200.orchestrator.assembly.expressions import (
    build_reduction_epilogue_transform,
    chain_value_transform,
)
from metellus_b200.orchestrator.assembly.extras import Extras, param_decl, pname
from metellus_b200.orchestrator.assembly.matmul import batch_stride_of
from metellus_b200.orchestrator.ir import ReductionOp, Tensor
from metellus_b200.orchestrator.kernel_group import FusionStrategy, KernelGroup
from metellus_b200.runtime.program import Kernel, NativeKernel

RED_THREADS = 256
SPLIT_MAX_ROWS = 148       # fewer rows than SMs ...
SPLIT_MIN_COLS = 1 << 16   # ... and long rows: split each row across many blocks


def assemble_split_reduction(decision: DecisionView, function_name: str | None) -> KernelGroup | None:
    """Few, long rows (a whole-tensor reduction viewed as (1, M*K) is the extreme
    case): the native split-row kernel of the backend (``mt_reduce_rows``), fp64
    partials combined deterministically. The reference runs such a reduction on a
    single threadgroup (assembly/reduction.py:105-106)."""
    from metellus_b200 import distributed

    anchor = decision.anchor
    combine = anchor.out.name in distributed.combined_outputs()
    if combine:
        # Every rank plans the same program on its own shard; they must all accept or
        # all reject the combine, or the accepting ranks would wait in the all-reduce
        # for ranks that raised. So each rank checks its shard and the verdicts are
        # exchanged on the host before anything is launched.
        problem = _combine_problem(decision)
        distributed.agree(problem, what=f"combined reduction {anchor.out.name!r}")
        return _combined_reduction(decision, function_name, anchor.input, *anchor.input.shape)
    if decision.strategy is not FusionStrategy.STANDALONE_REDUCTION or len(anchor.input.shape) != 2:
        return None
    src = anchor.input
    M, K = src.shape
    layout_ok = src.col_stride == 1 and (M == 1 or src.row_stride >= K)
    if M > SPLIT_MAX_ROWS or K < SPLIT_MIN_COLS or not layout_ok:
        return None
    ld = src.row_stride if M > 1 else K
    ctx = CodegenContext(function_name=function_name or f"reduce_split_{anchor.out.name}",
                         buffers=(param_decl(src.buffer_key), param_decl(anchor.out.buffer_key, writable=True)),
                         dims=("M", "K"), tg_x=256, tg_y=1)
    kernel = NativeKernel("mt_reduce_rows", (M, K, ld, anchor.op), ctx)
    return KernelGroup(kernel=kernel, bindings=(src.buffer_key, anchor.out.buffer_key), dims=(M, K),
                       grid=(0, M, 1), threads=(256, 1, 1), ops=decision.ops, strategy=decision.strategy,
                       pipe="native")


PARTIAL_KEY = "__mt_partial64"


def _combine_problem(decision: DecisionView) -> str | None:
    """Why this rank cannot combine the reduction across GPUs (None when it can).

    Only whole-tensor reductions combine: the input must be one row (``sum(X)`` is
    planned over the (1, M*K) view of the rank's rows). Per-row partials of several
    rows cannot be added element-wise across ranks, because row i of one rank's
    shard and row i of another's are different rows of the full tensor."""
    anchor = decision.anchor
    name = anchor.out.name
    if decision.strategy is not FusionStrategy.STANDALONE_REDUCTION or len(anchor.input.shape) != 2:
        return (f"reduction {name!r} is combined across GPUs, so it must be a standalone 2-D reduction "
                "(no fused prologue / epilogue)")
    src = anchor.input
    M, K = src.shape
    if M != 1:
        return (f"reduction {name!r} is combined across GPUs, so it must reduce the whole tensor: its input "
                f"must be a single row (view the shard as (1, M*K)), not {M} rows")
    if K < 1:
        return f"reduction {name!r} is combined across GPUs but this rank's shard is empty"
    if src.col_stride != 1:
        return f"reduction {name!r} is combined across GPUs but its input row is not contiguous"
    return None


def _combined_reduction(decision: DecisionView, function_name: str | None, src, M: int, K: int) -> KernelGroup:
    """Sharded whole-tensor reduction: this rank's fp64 partials (``mt_reduce_rows``
    with fp64 output, into scratch), then one NCCL all-reduce of the partials across
    the ranks that also writes the fp32 result (``mt_allreduce_f64``)."""
    anchor = decision.anchor
    ld = src.row_stride if M > 1 else K
    ctx = CodegenContext(function_name=function_name or f"reduce_allreduce_{anchor.out.name}",
                         buffers=(param_decl(src.buffer_key), param_decl(anchor.out.buffer_key, writable=True)),
                         dims=("M", "K"), tg_x=256, tg_y=1)
    kernel = NativeKernel("mt_reduce_rows+mt_allreduce_f64", (M, K, ld, anchor.op), ctx)
    return KernelGroup(kernel=kernel, bindings=(src.buffer_key, anchor.out.buffer_key), dims=(M, K),
                       grid=(0, M, 1), threads=(256, 1, 1), ops=decision.ops, strategy=decision.strategy,
                       pipe="native+nccl", scratch=((PARTIAL_KEY, 8 * M),))


COLRED_TARGET_BLOCKS = 148 * 8   # ~8 resident 256-thread blocks per SM
COLRED_MIN_CHUNK = 64            # reduced indices per split (8 per warp)


def column_reduction_plan(M: int, K: int) -> tuple[int, int]:
    """(column blocks, splits of the reduced axis) for an M-output, K-deep column
    reduction: enough blocks to fill the GPU, each split at least 64 indices deep."""
    colblocks = -(-M // COLRED_COLS)
    want = -(-COLRED_TARGET_BLOCKS // colblocks)
    splits = max(1, min(want, K // COLRED_MIN_CHUNK, 65535))
    return colblocks, splits


def assemble_column_reduction(decision: DecisionView, function_name: str | None) -> KernelGroup | None:
    """A reduction over a view with contiguous rows (``reduction(transpose(X))``):
    the coalesced column kernel (``ColumnReductionFragment``) with the prologue chain
    applied to each load and the epilogue chain to each result. None when the view
    is not of that layout."""
    anchor = decision.anchor
    src = decision.prologue_a[0].operands[0] if decision.prologue_a else anchor.input
    if not isinstance(src, Tensor) or len(src.shape) != 2 or src.row_stride != 1 or src.col_stride == 1:
        return None
    M, K = src.shape
    final_out = decision.epilogue[-1].out if decision.epilogue else anchor.out
    colblocks, splits = column_reduction_plan(M, K)
    part_key, ticket_key = f"__mt_colpart_{anchor.out.name}", f"__mt_colticket_{anchor.out.name}"
    scratch = ((part_key, 4 * splits * M), (ticket_key, 4 * colblocks)) if splits > 1 else ()
    extras = Extras(base_slots_by_key={src.buffer_key: 0, final_out.buffer_key: 1})
    pro = chain_value_transform(decision.prologue_a, row_var="row", col_var="idx", extras=extras,
                                base_slot=2) if decision.prologue_a else None
    epi = build_reduction_epilogue_transform(decision.epilogue) if decision.epilogue else None
    vec = M % 4 == 0 and src.col_stride % 4 == 0
    frag = ColumnReductionFragment(op=anchor.op, input_name=pname(src.buffer_key),
                                   output_name=pname(final_out.buffer_key), part_name=pname(part_key),
                                   ticket_name=pname(ticket_key), col_stride=src.col_stride, splits=splits,
                                   vec=vec, name="column_reduction", value_transform=pro, epilogue=epi)
    # parameter order = dispatch order: bindings (input, output, extras) then scratch
    params = (param_decl(src.buffer_key), param_decl(final_out.buffer_key, writable=True), *extras.buffers,
              *(param_decl(k, writable=True) for k, _ in scratch))
    fn = function_name or f"reduce_cols_{anchor.out.name}"
    ctx = CodegenContext(function_name=fn, buffers=params, dims=("M", "K"), tg_x=COLRED_WARPS * 32, tg_y=1,
                         threadgroup_decls=(f"smem float colred_sh[{COLRED_WARPS}][{COLRED_COLS}];",))
    return KernelGroup(kernel=Kernel(fragments=(frag,), ctx=ctx),
                       bindings=(src.buffer_key, final_out.buffer_key, *extras.bindings), dims=(M, K),
                       grid=(colblocks, splits, 1), threads=(COLRED_WARPS * 32, 1, 1), ops=decision.ops,
                       strategy=decision.strategy, scratch=scratch)


def assemble_reduction(decision: DecisionView, function_name: str | None) -> KernelGroup:
    anchor = decision.anchor
    assert isinstance(anchor, ReductionOp)
    split = assemble_split_reduction(decision, function_name)
    if split is not None:
        return split
    col = assemble_column_reduction(decision, function_name)
    if col is not None:
        return col
    src = decision.prologue_a[0].operands[0] if decision.prologue_a else anchor.input
    assert isinstance(src, Tensor)
    M, K = src.matrix_shape
    batch = src.batch
    final_out = decision.epilogue[-1].out if decision.epilogue else anchor.out
    extras = Extras(base_slots_by_key={src.buffer_key: 0, final_out.buffer_key: 1})
    pro = chain_value_transform(decision.prologue_a, row_var="row", col_var="idx", extras=extras,
                                base_slot=2) if decision.prologue_a else None
    epi = build_reduction_epilogue_transform(decision.epilogue) if decision.epilogue else None
    nt = RED_THREADS
    frags = (
        LastAxisReductionSetupFragment(rows_dim="M", name="reduction_setup"),
        LastAxisReductionComputeFragment(op=anchor.op, input_name=pname(src.buffer_key), scratch_name="scratch",
                                         reduce_dim="K", row_stride=str(src.row_stride), name="reduction_compute",
                                         tg_x=nt, col_stride=str(src.col_stride), value_transform=pro),
        StoreReductionResultFragment(output_name=pname(final_out.buffer_key), scratch_name="scratch",
                                     name="reduction_store", tg_x=nt, value_transform=epi),
    )
    bindings = (src.buffer_key, final_out.buffer_key, *extras.bindings)
    params = (param_decl(src.buffer_key), param_decl(final_out.buffer_key, writable=True),
              *extras.buffers)
    bstrides = (batch_stride_of(src), batch_stride_of(final_out), *extras.batch_strides)
    fn = function_name or f"reduce_{anchor.out.name}_fused"
    ctx = CodegenContext(function_name=fn, buffers=params, dims=("M", "K"), tg_x=nt, tg_y=1,
                         threadgroup_decls=(f"smem float scratch[{(nt + 31) // 32}];",),
                         batch_strides=bstrides if batch > 1 else ())
    return KernelGroup(kernel=Kernel(fragments=frags, ctx=ctx), bindings=bindings, dims=(M, K),
                       grid=(M, 1, batch), threads=(nt, 1, 1), ops=decision.ops, strategy=decision.strategy)
