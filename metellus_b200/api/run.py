"""End-to-end compile + run of an ``Operations`` program (reference: src/api/run.py).

``run(ops)`` = ``ops.build()`` -> ``fuse`` -> ``alias_group(assemble(v))`` ->
``schedule`` -> ``Runtime.run()``; returns ``RunResult(env, groups)``. With
``profile=True`` per-kernel device times (ms, CUDA events) land in env under ``t_0``,
``t_1``, ...

``compile_program(ops)`` stops before execution and returns the groups, so callers
that run the same program repeatedly (the bench, serving loops) plan and compile once.
"""

from __future__ import annotations

from typing import Any, NamedTuple

from metellus_b200.orchestrator.aliasing import alias_group
from metellus_b200.orchestrator.assembly import assemble
from metellus_b200.orchestrator.builder import Operations
from metellus_b200.orchestrator.fusion import fuse
from metellus_b200.orchestrator.kernel_group import KernelGroup
from metellus_b200.orchestrator.scheduler import schedule


class RunResult(NamedTuple):
    env: dict[str, Any]
    groups: tuple[KernelGroup, ...]


def compile_program(ops: Operations, *, b200: bool = True) -> tuple[KernelGroup, ...]:
    program = ops.build()
    vertices = fuse(program, b200=b200)
    return tuple(alias_group(assemble(v)) for v in vertices)


def run(ops: Operations, *, profile: bool = False, b200: bool = True) -> RunResult:
    groups = compile_program(ops, b200=b200)
    runtime = schedule(ops, groups, profile=profile)
    return RunResult(env=runtime.run(), groups=groups)
