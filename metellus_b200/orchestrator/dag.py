"""Producer / consumer view over an IR program (dag.py:46-76): validates SSA and
def-before-use, and exposes program inputs (read, never produced) and outputs
(produced, never read)."""

from __future__ import annotations

from collections import defaultdict
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
        cs = self.consumers_of.get(name, ())
        return cs[0] if len(cs) == 1 else None

    def topo_order(self) -> list[Op]:
        return list(self.program)


def build_dag(program: Program) -> DAG:
    producer_of: dict[str, Op] = {}
    consumer_lists: dict[str, list[Op]] = defaultdict(list)
    used: set[str] = set()
    for op in program:
        for t in op.inputs:
            consumer_lists[t.name].append(op)
            used.add(t.name)
        out_name = op.out.name
        if out_name in producer_of:
            raise ValueError(f"SSA violation: tensor {out_name!r} produced by two ops")
        if out_name in used:
            raise ValueError(
                f"def-after-use: tensor {out_name!r} consumed before it is defined "
                "(program must be in topological order)"
            )
        producer_of[out_name] = op
    produced = set(producer_of)
    return DAG(
        program=list(program),
        producer_of=producer_of,
        consumers_of={n: tuple(v) for n, v in consumer_lists.items()},
        inputs=frozenset(used - produced),
        outputs=frozenset(produced - used),
    )
