"""Producer / consumer index of an IR program (reference API: src/orchestrator/dag.py).

``build_dag`` walks the ops once, in program order, and checks the two rules the
rest of the compiler relies on: every tensor name is written by at most one op
(SSA), and no op writes a name that an earlier op already read (the program is in
topological order). It records who writes and who reads each name; program inputs
are the names read but never written, outputs the names written but never read.
"""

from __future__ import annotations

from dataclasses import dataclass

from metellus_b200.orchestrator.ir import Op, Program


@dataclass(frozen=True)
class DAG:
    program: Program
    producer_of: dict[str, Op]
    consumers_of: dict[str, tuple[Op, ...]]
    inputs: frozenset[str]
    outputs: frozenset[str]

    def unique_consumer(self, name: str) -> Op | None:
        """The only op reading ``name``, or None when zero or several ops read it."""
        readers = self.consumers_of.get(name, ())
        return readers[0] if len(readers) == 1 else None

    def topo_order(self) -> list[Op]:
        return list(self.program)


def build_dag(program: Program) -> DAG:
    writer: dict[str, Op] = {}
    readers: dict[str, list[Op]] = {}
    for op in program:
        for t in op.inputs:
            readers.setdefault(t.name, []).append(op)
        name = op.out.name
        if name in writer:
            raise ValueError(f"SSA violation: {name!r} is written by two ops")
        if name in readers:
            raise ValueError(f"def-after-use: {name!r} is read before the op that writes it "
                             "(ops must be listed in topological order)")
        writer[name] = op
    read, written = set(readers), set(writer)
    return DAG(program=list(program), producer_of=writer,
               consumers_of={n: tuple(ops) for n, ops in readers.items()},
               inputs=frozenset(read - written), outputs=frozenset(written - read))
