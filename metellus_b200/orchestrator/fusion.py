"""Fusion: IR program -> topo-ordered tuple of fused vertices (one kernel each).

Reference rules (src/orchestrator/fusion.py): the same eligibility predicates, the
same five rewrite passes in the same priority order (fusion.py:434-440), the same
saturation driver (first matching pass wins, restart from the top) and the same
budget gate (assemble every new vertex, compare its post-alias shared-memory bytes
with the cap, blacklist the offending signature and re-run, fusion.py:443-545). The
cap is the B200 one (``aliasing.TGMEM_CAP_BYTES``).

B200 passes run after the reference passes (so they never pre-empt a reference
fusion) and only when ``b200=True`` (the default):

* ``try_attention_fuse``  — matmul -> [scale] -> row softmax -> matmul, one kernel.
* ``try_row_fuse``        — merge reductions with the elementwise ops around them when
  everything lives on one row space (softmax, layernorm), one pass over HBM.
* ``try_elementwise_dag_fuse`` — merge elementwise vertices over one element space
  (multi-root DAGs such as config C2), one pass over HBM.

Views: a consumer that reads a *view* of a produced tensor (``row_max`` read as the
(M, 1) reshape ``row_max_2d``) depends on the producer of the view's storage owner.
The reference's vertex graph sees such reads as external inputs (graph.py:21-24);
the B200 passes resolve them through ``buffer_key`` so they can fuse across them.
"""

from __future__ import annotations

from metellus_b200.compute.elementwise import (
    BINARY_EXPRESSIONS,
    TERNARY_EXPRESSIONS,
    UNARY_EXPRESSIONS,
    BroadcastSpec,
)
from metellus_b200.orchestrator import aliasing
from metellus_b200.orchestrator.aliasing import TgmemOverflowError, compute_group_budget
from metellus_b200.orchestrator.graph import Graph, Vertex
from metellus_b200.orchestrator.ir import (
    ElementwiseOp,
    MatmulOp,
    Op,
    Program,
    ReductionOp,
    Scalar,
    ShapeOp,
    Tensor,
)

# Re-exported so callers (and tests) can monkeypatch the cap here, as with the
# reference's `orchestrator.fusion.TGMEM_CAP_BYTES`.
TGMEM_CAP_BYTES = aliasing.TGMEM_CAP_BYTES

# ---------------------------------------------------------------------------
# Eligibility predicates (fusion.py:68-115)
# ---------------------------------------------------------------------------


def _is_unary(op: ElementwiseOp) -> bool:
    return op.op in UNARY_EXPRESSIONS


def _is_binary(op: ElementwiseOp) -> bool:
    return op.op in BINARY_EXPRESSIONS


def _is_ternary(op: ElementwiseOp) -> bool:
    return op.op in TERNARY_EXPRESSIONS


def _is_lane_agnostic(op: ElementwiseOp) -> bool:
    if _is_ternary(op):
        return False
    return all(isinstance(o, Scalar) for o in op.operands[1:])


def _epilogue_eligible_matmul(elem: ElementwiseOp, primary_name: str) -> bool:
    if _is_ternary(elem):
        return False
    p = elem.operands[0]
    return isinstance(p, Tensor) and p.name == primary_name


def _prologue_eligible(elem: ElementwiseOp) -> bool:
    return _is_unary(elem) or _is_binary(elem)


def _reduction_epilogue_eligible(elem: ElementwiseOp) -> bool:
    if _is_unary(elem):
        return True
    if _is_binary(elem):
        return isinstance(elem.operands[1], Scalar)
    return False


def _anchor_of(vertex: Vertex) -> Op | None:
    for op in vertex.ops:
        if isinstance(op, (MatmulOp, ReductionOp)):
            return op
    return None


def _is_dual_gemm_vertex(vertex: Vertex) -> bool:
    """A vertex built by ``try_dual_gemm_fuse``; its tcgen05 template takes no
    prologues, so the reference prologue passes leave it alone."""
    if sum(isinstance(op, MatmulOp) for op in vertex.ops) != 2:
        return False
    from metellus_b200.orchestrator.assembly.decision import classify
    from metellus_b200.orchestrator.kernel_group import FusionStrategy

    return classify(vertex).strategy is FusionStrategy.DUAL_GEMM_EPILOGUE


def _is_chain_vertex(vertex: Vertex) -> bool:
    """An elementwise vertex whose ops form a linear chain (each op's primary operand is
    the previous op's output) -- the only elementwise shape the reference passes ever
    build, and the only one its prologue / epilogue templates evaluate. The B200
    elementwise-DAG pass builds other shapes; those are not absorbed into anchors."""
    if not _is_elementwise_vertex(vertex):
        return False
    for prev, cur in zip(vertex.ops, vertex.ops[1:]):
        p = cur.operands[0]
        if not (isinstance(p, Tensor) and p.name == prev.out.name):
            return False
    return True


def _is_elementwise_vertex(vertex: Vertex) -> bool:
    return len(vertex.ops) > 0 and all(isinstance(op, ElementwiseOp) for op in vertex.ops)


# ---------------------------------------------------------------------------
# Reference passes (fusion.py:145-393)
# ---------------------------------------------------------------------------


def try_elem_chain_fuse(graph: Graph, blacklist: frozenset[frozenset[int]]) -> Graph | None:
    """elem U -> elem V along V's head primary, U's tail having one consumer."""
    for u in graph.vertices:
        if not _is_elementwise_vertex(u):
            continue
        tail = u.ops[-1].out.name
        if tail not in u.outputs:
            continue
        cons = graph.consumers_of(tail)
        if len(cons) != 1:
            continue
        v = cons[0]
        if not _is_elementwise_vertex(v):
            continue
        head = v.ops[0]
        if _is_ternary(head):
            continue
        p = head.operands[0]
        if not isinstance(p, Tensor) or p.name != tail:
            continue
        if (u.op_ids | v.op_ids) in blacklist or not _views_local(u.ops + v.ops):
            continue
        try:
            return graph.replace(absorbed=(u, v), ops=u.ops + v.ops)
        except ValueError:  # not convex once view reads count as edges
            continue
    return None


def try_epilogue_absorb(graph: Graph, blacklist: frozenset[frozenset[int]]) -> Graph | None:
    """anchor A -> elem V (unique consumer) into A's epilogue."""
    for a in graph.vertices:
        anchor = _anchor_of(a)
        if anchor is None:
            continue
        tail = a.ops[-1].out.name
        if tail not in a.outputs:
            continue
        cons = graph.consumers_of(tail)
        if len(cons) != 1:
            continue
        v = cons[0]
        if not _is_chain_vertex(v):
            continue
        head = v.ops[0]
        if isinstance(anchor, MatmulOp):
            if not _epilogue_eligible_matmul(head, tail):
                continue
        else:
            if not _reduction_epilogue_eligible(head):
                continue
            p = head.operands[0]
            if not (isinstance(p, Tensor) and p.name == tail):
                continue
        if (a.op_ids | v.op_ids) in blacklist or not _views_local(a.ops + v.ops):
            continue
        try:
            return graph.replace(absorbed=(a, v), ops=a.ops + v.ops)
        except ValueError:  # not convex once view reads count as edges
            continue
    return None


def _anchor_boundary_input_names(anchor: Op, vertex: Vertex) -> set[str]:
    """Device-load sources of an anchor, walking back through absorbed prologues
    (fusion.py:396-426)."""
    if isinstance(anchor, MatmulOp):
        cands = [anchor.a.name, anchor.b.name]
    elif isinstance(anchor, ReductionOp):
        cands = [anchor.input.name]
    else:
        return set()
    pre = vertex.ops[: vertex.ops.index(anchor)]
    out: set[str] = set()
    for name in cands:
        cur = name
        while True:
            prod = next((op for op in pre if op.out.name == cur), None)
            if prod is None or not isinstance(prod, ElementwiseOp):
                break
            p = prod.operands[0]
            if not isinstance(p, Tensor):
                break
            cur = p.name
        out.add(cur)
    return out


def _view_is_local(view: Tensor, owner: Tensor) -> bool:
    """Whether a kernel that computes ``owner`` element by element can hand that value
    to a read of ``view`` at the same index: an identity view (same shape and strides),
    or a per-row vector in another shape ((M,) <-> (M, 1)). A transposed or reshaped
    view of a tensor produced in the same kernel reads elements another thread or
    block computes."""
    if (view.shape == owner.shape and view.row_stride == owner.row_stride
            and view.col_stride == owner.col_stride
            and (len(view.shape) != 3 or view.batch_stride == owner.batch_stride)):
        return True
    rv, ro = _row_space(view), _row_space(owner)
    return rv == ro and rv[1] is None


def _views_local(ops: tuple[Op, ...]) -> bool:
    """No op of a prospective kernel reads a non-local view (``_view_is_local``) of a
    tensor another op of the same kernel produces. The reference's fusion rules do not
    check this (its chain rule fuses ``y = t + transpose(t)`` with ``t``'s producer and
    reads ``t`` from memory that the same kernel is still writing); every merge here
    does."""
    produced = {op.out.name: op.out for op in ops}
    for op in ops:
        for t in op.inputs:
            owner = produced.get(t.buffer_key)
            if owner is not None and t.name != owner.name and not _view_is_local(t, owner):
                return False
    return True


def _merge_in_order(graph: Graph, *vertices: Vertex) -> tuple[Op, ...]:
    ops = [op for v in vertices for op in v.ops]
    return tuple(op for _, op in sorted(((graph.op_index[id(o)], o) for o in ops), key=lambda p: p[0]))


def try_prologue_absorb_single(graph: Graph, blacklist: frozenset[frozenset[int]]) -> Graph | None:
    """elem V -> anchor vertex A (unique consumer) into A's load transform."""
    for v in graph.vertices:
        if not _is_chain_vertex(v):
            continue
        tail = v.ops[-1].out.name
        if tail not in v.outputs:
            continue
        cons = graph.consumers_of(tail)
        if len(cons) != 1:
            continue
        a = cons[0]
        anchors = [op for op in a.ops if isinstance(op, (MatmulOp, ReductionOp))]
        if not anchors or _is_dual_gemm_vertex(a):
            continue
        names: set[str] = set()
        for anc in anchors:
            names |= _anchor_boundary_input_names(anc, a)
        if tail not in names:
            continue
        if not all(_prologue_eligible(op) for op in v.ops if isinstance(op, ElementwiseOp)):
            continue
        if (v.op_ids | a.op_ids) in blacklist or not _views_local(_merge_in_order(graph, v, a)):
            continue
        try:
            return graph.replace(absorbed=(v, a), ops=_merge_in_order(graph, v, a))
        except ValueError:  # not convex once view reads count as edges
            continue
    return None


def try_multi_producer_fuse(graph: Graph, blacklist: frozenset[frozenset[int]]) -> Graph | None:
    """Two pure matmul producers of one binary full-shape merge elem (fusion.py:259-318)."""
    for v in graph.vertices:
        if not _is_elementwise_vertex(v) or len(v.ops) != 1:
            continue
        elem = v.ops[0]
        if not _is_binary(elem) or elem.y_broadcast is not BroadcastSpec.NONE:
            continue
        x, y = elem.operands[0], elem.operands[1]
        if not (isinstance(x, Tensor) and isinstance(y, Tensor)):
            continue
        px, py = graph.producer_of(x.name), graph.producer_of(y.name)
        if px is None or py is None or px is py:
            continue
        if len(px.ops) != 1 or len(py.ops) != 1:
            continue
        ax, ay = px.ops[0], py.ops[0]
        if not (isinstance(ax, MatmulOp) and isinstance(ay, MatmulOp)):
            continue
        if len(graph.consumers_of(x.name)) != 1 or len(graph.consumers_of(y.name)) != 1:
            continue
        if ax.out.shape != ay.out.shape:
            continue
        if (px.op_ids | py.op_ids | v.op_ids) in blacklist or not _views_local(_merge_in_order(graph, px, py, v)):
            continue
        try:
            return graph.replace(absorbed=(px, py, v), ops=_merge_in_order(graph, px, py, v))
        except ValueError:  # not convex once view reads count as edges
            continue
    return None


def _should_recompute(elem: ElementwiseOp) -> bool:
    return _is_lane_agnostic(elem)


def try_prologue_absorb_multi(graph: Graph, blacklist: frozenset[frozenset[int]]) -> Graph | None:
    """Recompute a lane-agnostic elem inside each of its >= 2 anchor consumers."""
    for v in graph.vertices:
        if not _is_elementwise_vertex(v) or len(v.ops) != 1:
            continue
        elem = v.ops[0]
        if not _prologue_eligible(elem) or not _should_recompute(elem):
            continue
        out = elem.out.name
        if out not in v.outputs:
            continue
        cons = list(graph.consumers_of(out))
        if len(cons) < 2:
            continue
        ids: list[int] = []
        ok = True
        for c in cons:
            ac = _anchor_of(c)
            if ac is None or _is_dual_gemm_vertex(c) or out not in _anchor_boundary_input_names(ac, c):
                ok = False
                break
            ids.append(id(ac))
        if not ok:
            continue
        sig = v.op_ids | frozenset(o for c in cons for o in c.op_ids)
        if sig in blacklist:
            continue
        g = graph
        for aid in ids:
            cur = next(cv for cv in g.vertices if any(id(op) == aid for op in cv.ops))
            g = g.absorb_into(cur, v.ops)
        still = out in graph.program_outputs or any(out in g.reads(o) for o in g.vertices if o is not v)
        if not still:
            g = g.remove_vertex(v)
        return g
    return None


# ---------------------------------------------------------------------------
# B200 passes
# ---------------------------------------------------------------------------


def _owner_map(graph: Graph) -> dict[str, str]:
    """View name -> storage-owner name for views of tensors produced in the graph."""
    produced = {op.out.name for v in graph.vertices for op in v.ops}
    m: dict[str, str] = {}
    for v in graph.vertices:
        for op in v.ops:
            for t in op.inputs:
                if t.name not in produced and t.buffer_key in produced and t.buffer_key != t.name:
                    m[t.name] = t.buffer_key
    return m


def _resolved_inputs(v: Vertex, owners: dict[str, str]) -> set[str]:
    return {owners.get(n, n) for n in v.inputs}


def _edges(graph: Graph) -> list[tuple[Vertex, Vertex]]:
    """(producer, consumer) vertex pairs, view reads resolved to their owner."""
    owners = _owner_map(graph)
    prod: dict[str, Vertex] = {}
    for v in graph.vertices:
        for op in v.ops:
            prod[op.out.name] = v
    out = []
    seen = set()
    for c in graph.topo_sort():
        for n in sorted(_resolved_inputs(c, owners)):
            p = prod.get(n)
            if p is not None and p is not c and (id(p), id(c)) not in seen:
                seen.add((id(p), id(c)))
                out.append((p, c))
    return out


def _try_merge(graph: Graph, u: Vertex, v: Vertex) -> Graph | None:
    try:
        ops = _merge_in_order(graph, u, v)
        if not _views_local(ops):
            return None
        g = graph.replace(absorbed=(u, v), ops=ops)
    except ValueError:
        return None
    return g if _views_ordered(g) else None


def _views_ordered(graph: Graph) -> bool:
    """A merge must keep every view-read after its owner's producer in topo order."""
    owners = _owner_map(graph)
    order = graph.topo_sort()
    pos = {id(v): i for i, v in enumerate(order)}
    prod: dict[str, Vertex] = {}
    for v in graph.vertices:
        for op in v.ops:
            prod[op.out.name] = v
    for v in graph.vertices:
        for n in v.inputs:
            o = owners.get(n)
            if o is not None and prod[o] is not v and pos[id(prod[o])] > pos[id(v)]:
                return False
    return True


def _row_space(t: Tensor) -> tuple[int, int | None]:
    """(rows, cols) of a tensor in the row-resident sense: (B*M, N) for matrices,
    (B*M, None) for per-row vectors ((M,), (M, 1) views and batched forms)."""
    s = t.shape
    if len(s) == 1:
        return (s[0], None)
    if len(s) == 2:
        return (s[0], None) if s[1] == 1 else (s[0], s[1])
    B, M, N = s
    return (B * M, None) if N == 1 else (B * M, N)


def _row_vertex_space(v: Vertex) -> tuple[int, int] | None:
    """(rows, cols) if every op of ``v`` is a reduction / elementwise op over one row
    space with one column extent; None otherwise."""
    rows = None
    cols = None
    for op in v.ops:
        if isinstance(op, ReductionOp):
            r, c = _row_space(op.input)
        elif isinstance(op, ElementwiseOp):
            r, c = _row_space(op.out)
            for k, o in enumerate(op.operands[1:], start=1):
                if isinstance(o, Tensor):
                    mode = op.y_broadcast if k == 1 else op.cond_broadcast
                    if mode is BroadcastSpec.SCALAR and len(o.shape) == 3:
                        return None  # per-batch scalar: not expressible per row
        else:
            return None
        if rows is None:
            rows = r
        elif r != rows:
            return None
        if c is not None:
            if cols is None:
                cols = c
            elif c != cols:
                return None
    if rows is None or cols is None:
        return None
    return (rows, cols)


ROW_RESIDENT_MAX_COLS = 16384


def try_row_fuse(graph: Graph, blacklist: frozenset[frozenset[int]]) -> Graph | None:
    """Merge two row-compatible vertices joined by an edge when at least one holds a
    reduction: the fused vertex keeps each row on chip for the whole program."""
    for u, v in _edges(graph):
        su, sv = _row_vertex_space(u), _row_vertex_space(v)
        if su is None or sv is None or su != sv or su[1] > ROW_RESIDENT_MAX_COLS:
            continue
        if not any(isinstance(op, ReductionOp) for op in (*u.ops, *v.ops)):
            continue
        if (u.op_ids | v.op_ids) in blacklist:
            continue
        from metellus_b200.orchestrator.assembly.row_resident import row_program_check

        try:
            merged = _merge_in_order(graph, u, v)
        except ValueError:
            continue
        if row_program_check(merged) is not None:
            continue  # e.g. a reduction over a transposed view of a row it would hold
        g = _try_merge(graph, u, v)
        if g is not None:
            return g
    return None


def _ew_space(v: Vertex) -> tuple[int, ...] | None:
    if not _is_elementwise_vertex(v):
        return None
    shapes = {op.out.shape for op in v.ops}
    return next(iter(shapes)) if len(shapes) == 1 else None


def try_elementwise_dag_fuse(graph: Graph, blacklist: frozenset[frozenset[int]]) -> Graph | None:
    """Merge elementwise vertices over one element space joined by a full-shape edge."""
    for u, v in _edges(graph):
        su, sv = _ew_space(u), _ew_space(v)
        if su is None or su != sv:
            continue
        if (u.op_ids | v.op_ids) in blacklist:
            continue
        g = _try_merge(graph, u, v)
        if g is not None:
            return g
    return None


def _elementwise_region(graph: Graph, start: list[Vertex], shape: tuple[int, ...]) -> list[Vertex] | None:
    """Grow ``start`` by every elementwise vertex over ``shape`` that consumes a tensor
    the region produces; the region qualifies when exactly one of its tensors is read
    outside it (or is a program output) and that tensor is an elementwise result."""
    region = list(start)
    ids = {id(v) for v in region}
    grown = True
    while grown:
        grown = False
        for v in list(region):
            for name in v.outputs:
                for c in graph.consumers_of(name):
                    if id(c) in ids or not _is_elementwise_vertex(c):
                        continue
                    if any(op.out.shape != shape for op in c.ops):
                        continue
                    region.append(c)
                    ids.add(id(c))
                    grown = True
    produced = {op.out.name: op for v in region for op in v.ops}
    escaping = set()
    for name in produced:
        if name in graph.program_outputs or any(id(c) not in ids for c in graph.consumers_of(name)):
            escaping.add(name)
    if len(escaping) != 1:
        return None
    final = produced[next(iter(escaping))]
    return region if isinstance(final, ElementwiseOp) else None


def try_dual_gemm_fuse(graph: Graph, blacklist: frozenset[frozenset[int]]) -> Graph | None:
    """Two matmuls reading the same A whose outputs meet in an elementwise DAG with a
    single result (a gated MLP's ``act(H @ W1 + b1) * (H @ W3)``): one tcgen05 kernel
    streams A once into two TMEM accumulators and evaluates the whole DAG in its
    epilogue, so neither product nor any intermediate reaches HBM. Runs before the
    reference passes, which would otherwise split the DAG into epilogues, separate
    elementwise kernels and a prologue of the next matmul."""
    from metellus_b200.orchestrator.assembly.tc_matmul import dual_gemm_eligible

    mms = [v for v in graph.vertices if len(v.ops) == 1 and isinstance(v.ops[0], MatmulOp)]
    for i, p0 in enumerate(mms):
        for p1 in mms[i + 1:]:
            a0, a1 = p0.ops[0], p1.ops[0]
            if not dual_gemm_eligible(a0, a1):
                continue
            if any(graph.consumers_of(a.out.name) == () or a.out.name in graph.program_outputs
                   for a in (a0, a1)):
                continue
            region = _elementwise_region(graph, [p0, p1], a0.out.shape)
            if region is None or len(region) == 2:
                continue
            if frozenset(o for v in region for o in v.op_ids) in blacklist:
                continue
            try:
                ops = _merge_in_order(graph, *region)
                if not _views_local(ops):
                    continue
                g = graph.replace(absorbed=tuple(region), ops=ops)
            except ValueError:
                continue
            if _views_ordered(g):
                return g
    return None


def try_attention_fuse(graph: Graph, blacklist: frozenset[frozenset[int]]) -> Graph | None:
    from metellus_b200.orchestrator.assembly.attention import match_attention

    return match_attention(graph, blacklist)


B200_FIRST_PASSES = (try_dual_gemm_fuse,)
REFERENCE_PASSES = (
    try_elem_chain_fuse,
    try_multi_producer_fuse,
    try_epilogue_absorb,
    try_prologue_absorb_single,
    try_prologue_absorb_multi,
)
B200_PASSES = (
    try_attention_fuse,
    try_row_fuse,
    try_elementwise_dag_fuse,
)
_PASSES = B200_FIRST_PASSES + REFERENCE_PASSES + B200_PASSES


# ---------------------------------------------------------------------------
# Driver (fusion.py:443-545)
# ---------------------------------------------------------------------------


def _cap() -> int:
    return TGMEM_CAP_BYTES


def _check_primitive_budgets(graph: Graph) -> None:
    from metellus_b200.orchestrator.assembly import assemble

    cap = _cap()
    for v in graph.vertices:
        b = compute_group_budget(assemble(v))
        if b.size_bytes > cap:
            names = ", ".join(f"{type(op).__name__}({op.out.name})" for op in v.ops)
            raise TgmemOverflowError(
                f"primitive vertex [{names}] needs {b.size_bytes}B of shared memory; cap is "
                f"{cap}B. No fusion can shrink a single op — reduce its tile shape or pick a "
                "register-resident strategy."
            )


def _fits_budget(old: Graph, new: Graph) -> bool:
    from metellus_b200.orchestrator.assembly import assemble

    cap = _cap()
    old_ids = {id(v) for v in old.vertices}
    for v in new.vertices:
        if id(v) in old_ids:
            continue
        if compute_group_budget(assemble(v)).size_bytes > cap:
            return False
    return True


def _modified_signature(old: Graph, new: Graph) -> frozenset[int]:
    old_ids = {id(v) for v in old.vertices}
    sig: frozenset[int] = frozenset()
    for v in new.vertices:
        if id(v) not in old_ids:
            sig = sig | v.op_ids
    return sig


def _fuse_once(program: Program, blacklist: frozenset[frozenset[int]], passes) -> tuple[tuple[Vertex, ...], frozenset[int] | None]:
    graph = Graph.from_program(program)
    _check_primitive_budgets(graph)
    while True:
        for pass_fn in passes:
            new = pass_fn(graph, blacklist)
            if new is None:
                continue
            if not _fits_budget(graph, new):
                return new.topo_sort(), _modified_signature(graph, new)
            graph = new
            break
        else:
            return _ordered(graph), None


def _ordered(graph: Graph) -> tuple[Vertex, ...]:
    """Topological order that also respects view reads (a vertex reading a view of
    another vertex's output runs after it)."""
    order = list(graph.topo_sort())
    owners = _owner_map(graph)
    if not owners:
        return tuple(order)
    prod: dict[str, Vertex] = {}
    for v in graph.vertices:
        for op in v.ops:
            prod[op.out.name] = v
    changed = True
    while changed:
        changed = False
        pos = {id(v): i for i, v in enumerate(order)}
        for v in list(order):
            for n in v.inputs:
                o = owners.get(n)
                if o is None:
                    continue
                p = prod[o]
                if p is not v and pos[id(p)] > pos[id(v)]:
                    order.remove(p)
                    order.insert(pos[id(v)], p)
                    changed = True
                    break
            if changed:
                break
    return tuple(order)


def fuse(program: Program, *, b200: bool = True) -> tuple[Vertex, ...]:
    """Saturate the pass set under the budget gate; returns vertices in dispatch
    order. ``b200=False`` runs the reference pass set only (used to check plans
    against the reference's own fuser)."""
    passes = _PASSES if b200 else REFERENCE_PASSES
    blacklist: frozenset[frozenset[int]] = frozenset()
    while True:
        vertices, straw = _fuse_once(program, blacklist, passes)
        if straw is None:
            return vertices
        blacklist = blacklist | {straw}
