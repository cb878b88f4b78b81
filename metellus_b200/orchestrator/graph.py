"""Vertex graph over an IR program — the substrate the fusion passes rewrite.

Same contract as the reference (src/orchestrator/graph.py:40-428): immutable
``Graph`` of ``Vertex`` (ops + boundary inputs/outputs); ``replace`` collapses a
convex vertex set, ``absorb_into`` replicates producer ops into one consumer
(recompute), ``remove_vertex`` drops a dead producer, ``topo_sort`` is deterministic
(ties broken by the earliest contained op's IR position), ``check_dependencies``
verifies every producer->consumer edge of the original program is still respected.
"""

from __future__ import annotations

from dataclasses import dataclass, field

from metellus_b200.orchestrator.ir import Op, Program


@dataclass(frozen=True)
class Vertex:
    ops: tuple[Op, ...]
    inputs: tuple[str, ...]
    outputs: tuple[str, ...]

    @property
    def is_primitive(self) -> bool:
        return len(self.ops) == 1

    @property
    def op_ids(self) -> frozenset[int]:
        return frozenset(id(op) for op in self.ops)


@dataclass(frozen=True)
class Graph:
    vertices: tuple[Vertex, ...]
    op_index: dict[int, int]
    program_outputs: frozenset[str]
    # view name -> storage owner, for every view an op reads (transpose / reshape): a
    # vertex reading a view depends on, and keeps materialised, the owner's producer
    view_owner: dict[str, str] = field(default_factory=dict, compare=False)

    @classmethod
    def from_program(
        cls, program: Program, *, program_outputs: frozenset[str] | None = None
    ) -> Graph:
        op_index = {id(op): i for i, op in enumerate(program)}
        produced = {op.out.name for op in program}
        view_owner = {t.name: t.buffer_key for op in program for t in op.inputs if t.name != t.buffer_key}
        used = {t.name for op in program for t in op.inputs}
        # program outputs as the reference defines them: produced and never read by name
        # (a tensor read only through a view is still an output)
        outs = frozenset(produced - used) if program_outputs is None else frozenset(program_outputs)
        used |= set(view_owner.values())
        vertices = []
        for op in program:
            name = op.out.name
            visible = name in used or name in outs
            vertices.append(Vertex(ops=(op,), inputs=tuple(t.name for t in op.inputs),
                                   outputs=(name,) if visible else ()))
        return cls(vertices=tuple(vertices), op_index=op_index, program_outputs=outs, view_owner=view_owner)

    # -- rewrites ------------------------------------------------------------------

    def _with(self, vertices: tuple[Vertex, ...]) -> Graph:
        return Graph(vertices=vertices, op_index=self.op_index, program_outputs=self.program_outputs,
                     view_owner=self.view_owner)

    def reads(self, v: Vertex) -> set[str]:
        """Names ``v`` reads: its inputs plus the storage owner of every view among
        them."""
        return set(v.inputs) | {self.view_owner[n] for n in v.inputs if n in self.view_owner}

    def replace(self, absorbed: tuple[Vertex, ...], ops: tuple[Op, ...]) -> Graph:
        """Collapse ``absorbed`` into one vertex holding ``ops`` (graph.py:118-212)."""
        if not absorbed:
            raise ValueError("replace: absorbed set is empty")
        members = {id(v) for v in self.vertices}
        taken: set[int] = set()
        for v in absorbed:
            if id(v) not in members:
                raise ValueError("replace: absorbed contains a vertex not in this graph")
            if id(v) in taken:
                raise ValueError("replace: absorbed contains duplicate vertices")
            taken.add(id(v))
        if frozenset(id(o) for v in absorbed for o in v.ops) != frozenset(id(o) for o in ops):
            raise ValueError("replace: ops does not match the union of absorbed vertices' ops")
        pos = [self.op_index[id(o)] for o in ops]
        if pos != sorted(pos):
            raise ValueError("replace: ops must be in original-IR program order")

        inside = {o.out.name for o in ops}
        still_read: set[str] = set()
        for v in self.vertices:
            if id(v) not in taken:
                still_read.update(self.reads(v))
        read_by_absorbed: set[str] = set()
        for v in absorbed:
            read_by_absorbed.update(v.inputs)
        merged = Vertex(
            ops=tuple(ops),
            inputs=tuple(sorted(read_by_absorbed - inside)),
            outputs=tuple(sorted(n for n in inside if n in still_read or n in self.program_outputs)),
        )
        out: list[Vertex] = []
        placed = False
        for v in self.vertices:
            if id(v) in taken:
                if not placed:
                    out.append(merged)
                    placed = True
            else:
                out.append(v)
        g = self._with(tuple(out))
        try:
            g.topo_sort()
        except ValueError:
            raise ValueError(
                "replace: collapsing the absorbed set would introduce a cycle — the "
                "absorbed vertices are not convex in the dependency order"
            ) from None
        return g

    def absorb_into(self, consumer: Vertex, additional_ops: tuple[Op, ...]) -> Graph:
        """Replicate ``additional_ops`` into ``consumer`` (graph.py:335-390)."""
        if all(v is not consumer for v in self.vertices):
            raise ValueError("absorb_into: consumer not in this graph")
        if not additional_ops:
            raise ValueError("absorb_into: additional_ops is empty")
        merged_ops = tuple(
            op for _, op in sorted(((self.op_index[id(o)], o) for o in (*additional_ops, *consumer.ops)),
                                   key=lambda p: p[0])
        )
        extra_in = {t.name for o in additional_ops for t in o.inputs}
        extra_out = {o.out.name for o in additional_ops}
        nv = Vertex(ops=merged_ops,
                    inputs=tuple(sorted((set(consumer.inputs) | extra_in) - extra_out)),
                    outputs=consumer.outputs)
        g = self._with(tuple(nv if v is consumer else v for v in self.vertices))
        try:
            g.topo_sort()
        except ValueError:
            raise ValueError(
                "absorb_into: result is cyclic (additional_ops' inputs transitively "
                "depend on the consumer's outputs)"
            ) from None
        return g

    def remove_vertex(self, vertex: Vertex) -> Graph:
        """Drop a producer whose outputs nobody reads any more (graph.py:392-416)."""
        if all(v is not vertex for v in self.vertices):
            raise ValueError("remove_vertex: vertex not in this graph")
        for name in vertex.outputs:
            if name in self.program_outputs:
                raise ValueError(f"remove_vertex: output {name!r} is a program output; cannot remove")
            for other in self.vertices:
                if other is not vertex and name in self.reads(other):
                    raise ValueError(f"remove_vertex: output {name!r} still consumed by another vertex")
        return self._with(tuple(v for v in self.vertices if v is not vertex))

    # -- queries ---------------------------------------------------------------------

    def topo_sort(self) -> tuple[Vertex, ...]:
        """Kahn's algorithm; the ready set is ordered by each vertex's first IR op."""
        producer: dict[str, int] = {}
        for i, v in enumerate(self.vertices):
            for name in v.outputs:
                producer[name] = i
        n = len(self.vertices)
        succ: list[set[int]] = [set() for _ in range(n)]
        indeg = [0] * n
        for i, v in enumerate(self.vertices):
            deps = {producer[nm] for nm in self.reads(v) if nm in producer and producer[nm] != i}
            indeg[i] = len(deps)
            for d in deps:
                succ[d].add(i)
        first = [min(self.op_index[id(o)] for o in v.ops) for v in self.vertices]
        ready = sorted((i for i in range(n) if indeg[i] == 0), key=lambda i: first[i])
        order: list[int] = []
        while ready:
            i = ready.pop(0)
            order.append(i)
            for s in succ[i]:
                indeg[s] -= 1
                if indeg[s] == 0:
                    ready.append(s)
            ready.sort(key=lambda j: first[j])
        if len(order) != n:
            raise ValueError("graph contains a cycle")
        return tuple(self.vertices[i] for i in order)

    def flatten(self) -> tuple[Op, ...]:
        return tuple(op for v in self.topo_sort() for op in v.ops)

    def check_dependencies(self, original: Program) -> None:
        """Every original data edge must have a producer occurrence before each
        consumer occurrence in ``flatten()`` (graph.py:264-324)."""
        flat = self.flatten()
        positions: dict[int, list[int]] = {}
        for i, op in enumerate(flat):
            positions.setdefault(id(op), []).append(i)
        orig_ids = {id(op) for op in original}
        missing = orig_ids - set(positions)
        if missing:
            names = [f"{type(op).__name__}({op.out.name})" for op in original if id(op) in missing]
            raise ValueError(f"graph missing IR ops: {names}")
        if set(positions) - orig_ids:
            raise ValueError(
                "graph contains ops not in original IR — replace() received ops that "
                "don't belong to this Program"
            )
        producer_of = {op.out.name: op for op in original}
        for op in original:
            for t in op.inputs:
                prod = producer_of.get(t.name)
                if prod is None:
                    continue
                pp = positions[id(prod)]
                for c in positions[id(op)]:
                    if not any(p < c for p in pp):
                        raise ValueError(
                            f"dependency violated: {type(prod).__name__}({prod.out.name}) has no "
                            f"occurrence before {type(op).__name__}({op.out.name}) at flatten-pos "
                            f"{c} (consumed via tensor {t.name!r})"
                        )

    def preserves_dependencies(self, original: Program) -> bool:
        try:
            self.check_dependencies(original)
        except ValueError:
            return False
        return True

    def producer_of(self, name: str) -> Vertex | None:
        for v in self.vertices:
            if name in v.outputs:
                return v
        return None

    def consumers_of(self, name: str) -> tuple[Vertex, ...]:
        """Vertices that read ``name`` directly or through a view of it."""
        return tuple(v for v in self.topo_sort() if name in self.reads(v))
