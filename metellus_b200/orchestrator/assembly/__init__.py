"""Assemble a fused vertex into a ``KernelGroup`` (reference: assembly/__init__.py:59-74):
classify, then dispatch to the per-strategy template."""

from __future__ import annotations

from metellus_b200.orchestrator.assembly.decision import classify
from metellus_b200.orchestrator.graph import Vertex
from metellus_b200.orchestrator.kernel_group import FusionStrategy, KernelGroup

_MATMUL = {
    FusionStrategy.STANDALONE_MATMUL,
    FusionStrategy.MATMUL_EPILOGUE_TG,
    FusionStrategy.MATMUL_EPILOGUE_REGISTER,
    FusionStrategy.ELEMENTWISE_PROLOGUE_MATMUL,
}
_REDUCTION = {
    FusionStrategy.STANDALONE_REDUCTION,
    FusionStrategy.REDUCTION_EPILOGUE,
    FusionStrategy.ELEMENTWISE_PROLOGUE_REDUCTION,
}
_ELEMENTWISE = {
    FusionStrategy.STANDALONE_ELEMENTWISE,
    FusionStrategy.ELEMENTWISE_CHAIN,
    FusionStrategy.ELEMENTWISE_DAG,
}
_MULTI = {FusionStrategy.MULTI_PRODUCER_CONVERGENT, FusionStrategy.DIAMOND_SHARED,
          FusionStrategy.DUAL_GEMM_EPILOGUE}


def assemble(vertex: Vertex, *, function_name: str | None = None) -> KernelGroup:
    from metellus_b200.orchestrator.assembly.attention import assemble_attention
    from metellus_b200.orchestrator.assembly.elementwise import assemble_elementwise
    from metellus_b200.orchestrator.assembly.matmul import assemble_matmul
    from metellus_b200.orchestrator.assembly.multi_anchor import assemble_multi_anchor
    from metellus_b200.orchestrator.assembly.reduction import assemble_reduction
    from metellus_b200.orchestrator.assembly.row_resident import assemble_row_resident
    from metellus_b200.orchestrator.assembly.shape import assemble_shape

    d = classify(vertex)
    s = d.strategy
    if s in _MATMUL:
        return assemble_matmul(d, function_name)
    if s in _REDUCTION:
        return assemble_reduction(d, function_name)
    if s in _ELEMENTWISE:
        return assemble_elementwise(d, function_name)
    if s is FusionStrategy.STANDALONE_SHAPE:
        return assemble_shape(d, function_name)
    if s in _MULTI:
        return assemble_multi_anchor(d, function_name)
    if s is FusionStrategy.ROW_RESIDENT:
        return assemble_row_resident(d, function_name)
    if s is FusionStrategy.FUSED_ATTENTION:
        return assemble_attention(d, function_name)
    raise ValueError(f"unknown strategy {s!r}")


__all__ = ["assemble"]
