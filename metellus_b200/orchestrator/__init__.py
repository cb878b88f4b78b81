"""Orchestrator: IR, builder, DAG view and vertex graph (reference:
src/orchestrator/__init__.py). ``fuse`` / ``assemble`` / ``schedule`` live in their
submodules."""

from metellus_b200.compute.elementwise import BroadcastSpec
from metellus_b200.orchestrator.builder import Operations
from metellus_b200.orchestrator.dag import DAG, build_dag
from metellus_b200.orchestrator.graph import Graph, Vertex
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

__all__ = ["BroadcastSpec", "DAG", "ElementwiseOp", "Graph", "Layout", "MatmulOp", "Op", "OperandValue",
           "Operations", "Program", "ReductionOp", "Scalar", "ShapeOp", "Tensor", "Vertex", "build_dag"]
