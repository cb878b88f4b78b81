"""Seeded random programs (the planner property tests' generator, finite-valued
variant) run end to end on the GPU and compared with the fp64 oracle: every
materialised output, matmul tolerance where a matmul feeds it, elementwise tolerance
otherwise. Exercises fusion plans no hand-written case covers."""

from __future__ import annotations

import numpy as np
import pytest

from metellus_b200 import run
from metellus_b200.orchestrator.ir import MatmulOp
from oracle.ir_eval import evaluate
from tests.test_plan_properties import random_program
from tests.tolerances import assert_elementwise_close, assert_matmul_close

pytestmark = pytest.mark.gpu


def _depends_on_matmul(ops, name: str) -> bool:
    prog = ops.build()
    producer = {op.out.name: op for op in prog}
    owner = {t.name: t.buffer_key for t in ops.tensors.values()}
    stack, seen = [name], set()
    while stack:
        n = stack.pop()
        n = owner.get(n, n)
        if n in seen or n not in producer:
            continue
        seen.add(n)
        op = producer[n]
        if isinstance(op, MatmulOp):
            return True
        stack.extend(t.name for t in op.inputs)
    return False


@pytest.mark.parametrize("large", [False, True], ids=["simt", "tcgen05"])
@pytest.mark.parametrize("seed", range(20))
def test_random_program_matches_oracle(cuda_device, seed, large):
    ops = random_program(seed * 7919 + 11, safe=True, large=large)
    res = run(ops)
    r64 = evaluate(ops, np.float64)
    r32 = evaluate(ops, np.float32)
    checked = 0
    for name, val in res.env.items():
        if name.startswith("t_") and name[2:].isdigit() or name not in r64:
            continue
        if _depends_on_matmul(ops, name):
            assert_matmul_close(val, r64[name], r32[name], what=f"seed {seed}: {name}")
        else:
            assert_elementwise_close(val, r64[name], rel=2e-6, abs_=1e-6, what=f"seed {seed}: {name}")
        checked += 1
    assert checked >= 1
