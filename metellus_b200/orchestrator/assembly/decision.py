"""Classification: Vertex -> DecisionView (reference: assembly/decision.py:52-212).

The reference shapes (single matmul / reduction anchor with a traced prologue chain
and an epilogue chain, two-anchor merge, elementwise chain, shape copy) classify
exactly as in the reference. Vertices that only the B200 passes build classify into
the B200 strategies: a non-chain elementwise DAG -> ELEMENTWISE_DAG; reductions mixed
with full-row elementwise ops -> ROW_RESIDENT; matmul + reductions -> FUSED_ATTENTION;
two matmuls sharing A with an elementwise DAG over both -> DUAL_GEMM_EPILOGUE.
"""

from __future__ import annotations

from dataclasses import dataclass

from metellus_b200.compute.elementwise import TERNARY_EXPRESSIONS
from metellus_b200.orchestrator.graph import Vertex
from metellus_b200.orchestrator.ir import (
    ElementwiseOp,
    MatmulOp,
    Op,
    ReductionOp,
    Scalar,
    ShapeOp,
    Tensor,
)
from metellus_b200.orchestrator.kernel_group import FusionStrategy


@dataclass
class DecisionView:
    strategy: FusionStrategy
    anchor: MatmulOp | ReductionOp | None = None
    prologue_a: tuple[ElementwiseOp, ...] = ()
    prologue_b: tuple[ElementwiseOp, ...] = ()
    epilogue: tuple[ElementwiseOp, ...] = ()
    chain_only: tuple[ElementwiseOp, ...] = ()
    shape_op: ShapeOp | None = None
    ops: tuple[Op, ...] = ()
    anchors: tuple[MatmulOp, ...] = ()
    merge_elem: ElementwiseOp | None = None
    shared_a: bool = False
    prologues_a: tuple[tuple[ElementwiseOp, ...], ...] = ()
    prologues_b: tuple[tuple[ElementwiseOp, ...], ...] = ()
    # Boundary of the vertex (which tensors must be materialised).
    outputs: tuple[str, ...] = ()


def is_lane_agnostic_pred(op: ElementwiseOp) -> bool:
    """Every secondary operand is a Scalar (decision.py:374-383)."""
    if op.op in TERNARY_EXPRESSIONS:
        return False
    return all(isinstance(o, Scalar) for o in op.operands[1:])


def trace_prologue(target_name: str, candidates: tuple[Op, ...]) -> tuple[ElementwiseOp, ...]:
    """Walk back from ``target_name`` through elementwise producers along their
    primary operands; returns the chain head-first (decision.py:352-371)."""
    chain: list[ElementwiseOp] = []
    current = target_name
    while True:
        producer = next((op for op in candidates if op.out.name == current), None)
        if not isinstance(producer, ElementwiseOp):
            break
        chain.append(producer)
        primary = producer.operands[0]
        if not isinstance(primary, Tensor):
            break
        current = primary.name
    chain.reverse()
    return tuple(chain)


def is_linear_chain(ops: tuple[ElementwiseOp, ...]) -> bool:
    """True when each op's primary operand is the previous op's output."""
    for prev, cur in zip(ops, ops[1:]):
        p = cur.operands[0]
        if not (isinstance(p, Tensor) and p.name == prev.out.name):
            return False
    return True


def classify(vertex: Vertex) -> DecisionView:
    ops = vertex.ops
    outs = tuple(vertex.outputs)
    shape_op = next((op for op in ops if isinstance(op, ShapeOp)), None)
    if shape_op is not None:
        assert len(ops) == 1, "ShapeOp must be standalone"
        return DecisionView(strategy=FusionStrategy.STANDALONE_SHAPE, shape_op=shape_op, ops=ops,
                            outputs=outs)

    matmuls = tuple(op for op in ops if isinstance(op, MatmulOp))
    reductions = tuple(op for op in ops if isinstance(op, ReductionOp))

    if matmuls and reductions:
        return DecisionView(strategy=FusionStrategy.FUSED_ATTENTION, anchors=matmuls, ops=ops,
                            outputs=outs)

    if len(matmuls) >= 2:
        assert len(matmuls) == 2, "multi-anchor vertex must have exactly 2 matmul anchors"
        a0, a1 = matmuls
        i0, i1 = ops.index(a0), ops.index(a1)
        pre0 = tuple(op for op in ops[:i0] if isinstance(op, ElementwiseOp))
        pre1 = tuple(op for op in ops[:i1] if isinstance(op, ElementwiseOp))
        pa = (trace_prologue(a0.a.name, pre0), trace_prologue(a1.a.name, pre1))
        pb = (trace_prologue(a0.b.name, pre0), trace_prologue(a1.b.name, pre1))
        absorbed = {id(op) for ch in (*pa, *pb) for op in ch}
        post = tuple(op for op in ops if isinstance(op, ElementwiseOp) and id(op) not in absorbed)
        shared = a0.a.name == a1.a.name and a0.a.shape == a1.a.shape and not pa[0] and not pa[1]
        if len(post) > 1 or (post and ops.index(post[0]) < max(i0, i1)):
            # B200 dual GEMM: both anchors read one A; an elementwise DAG over the two
            # accumulators (and other full-shape / broadcast tensors) is the epilogue.
            assert shared and not absorbed and len(outs) == 1, \
                "dual-GEMM vertex: shared A, no prologues, one output"
            final = next(op for op in post if op.out.name == outs[0])
            return DecisionView(strategy=FusionStrategy.DUAL_GEMM_EPILOGUE, anchors=matmuls, merge_elem=final,
                                shared_a=True, prologues_a=((), ()), prologues_b=((), ()), epilogue=post,
                                ops=ops, outputs=outs)
        assert len(post) == 1, "multi-anchor vertex has exactly one merge elem"
        merge = post[0]
        return DecisionView(
            strategy=FusionStrategy.DIAMOND_SHARED if shared else FusionStrategy.MULTI_PRODUCER_CONVERGENT,
            anchors=matmuls, merge_elem=merge, shared_a=shared, prologues_a=pa, prologues_b=pb,
            ops=ops, outputs=outs,
        )

    anchor = matmuls[0] if matmuls else (reductions[0] if reductions else None)
    if anchor is None:
        chain = tuple(op for op in ops if isinstance(op, ElementwiseOp))
        assert len(chain) == len(ops)
        if len(chain) == 1:
            strategy = FusionStrategy.STANDALONE_ELEMENTWISE
        elif is_linear_chain(chain):
            strategy = FusionStrategy.ELEMENTWISE_CHAIN
        else:
            strategy = FusionStrategy.ELEMENTWISE_DAG
        return DecisionView(strategy=strategy, chain_only=chain, ops=ops, outputs=outs)

    idx = ops.index(anchor)
    pre = ops[:idx]
    post = tuple(op for op in ops[idx + 1:] if isinstance(op, ElementwiseOp))

    if isinstance(anchor, MatmulOp):
        final = post[-1].out.name if post else anchor.out.name
        extra = set(outs) - {final}
        assert not extra, f"matmul vertex must materialise only its final output; also needs {sorted(extra)}"
        pa = trace_prologue(anchor.a.name, pre)
        pb = trace_prologue(anchor.b.name, pre)
        if post and all(is_lane_agnostic_pred(e) for e in post):
            strategy = FusionStrategy.MATMUL_EPILOGUE_REGISTER
        elif post:
            strategy = FusionStrategy.MATMUL_EPILOGUE_TG
        elif pa or pb:
            strategy = FusionStrategy.ELEMENTWISE_PROLOGUE_MATMUL
        else:
            strategy = FusionStrategy.STANDALONE_MATMUL
        return DecisionView(strategy=strategy, anchor=anchor, prologue_a=pa, prologue_b=pb,
                            epilogue=post, ops=ops, outputs=outs)

    prologue = trace_prologue(anchor.input.name, pre)
    reference_shaped = (
        len(reductions) == 1
        and {id(o) for o in pre} == {id(o) for o in prologue}
        and (not post or (isinstance(post[0].operands[0], Tensor)
                          and post[0].operands[0].name == anchor.out.name
                          and is_linear_chain(post)))
        and all(len(e.out.matrix_shape) == 1 for e in post)
        # the reference reduction templates store only the final value; a vertex that
        # must also materialise a prologue or intermediate value (built by the B200 row
        # pass when that value has another consumer) runs row-resident
        and set(outs) <= {(post[-1].out.name if post else anchor.out.name)}
    )
    if not reference_shaped:
        return DecisionView(strategy=FusionStrategy.ROW_RESIDENT, ops=ops, outputs=outs)
    if prologue:
        strategy = FusionStrategy.ELEMENTWISE_PROLOGUE_REDUCTION
    elif post:
        strategy = FusionStrategy.REDUCTION_EPILOGUE
    else:
        strategy = FusionStrategy.STANDALONE_REDUCTION
    return DecisionView(strategy=strategy, anchor=anchor, prologue_a=prologue, epilogue=post,
                        ops=ops, outputs=outs)
