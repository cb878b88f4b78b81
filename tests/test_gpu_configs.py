"""GPU parity: the five benchmark programs (reduced shapes) through the public ``run``
API on the B200, checked against the CPU oracle (fp64 ground truth, fp32 reference
semantics). Tolerances: tests/tolerances.py."""

from __future__ import annotations

import numpy as np
import pytest

from metellus_b200 import configs, run
from metellus_b200.orchestrator.kernel_group import FusionStrategy
from oracle.ir_eval import evaluate
from tests.tolerances import assert_elementwise_close, assert_matmul_close

pytestmark = pytest.mark.gpu


def _check_all_outputs(key, ops, env, matmul: bool, tol_rel=1e-6, tol_abs=2e-7):
    r64 = evaluate(ops, np.float64)
    r32 = evaluate(ops, np.float32)
    out = configs.CONFIGS[key].output
    assert out in env, f"{key}: output {out!r} not materialised"
    if matmul:
        assert_matmul_close(env[out], r64[out], r32[out], what=key)
    else:
        assert_elementwise_close(env[out], r64[out], rel=tol_rel, abs_=tol_abs, what=key)
    # every other materialised tensor must agree as well
    for name, val in env.items():
        if name.startswith("t_") or name == out or name not in r64:
            continue
        if matmul:
            assert_matmul_close(val, r64[name], r32[name], what=f"{key}:{name}")
        else:
            assert_elementwise_close(val, r64[name], rel=1e-5, abs_=1e-6, what=f"{key}:{name}")


def test_c2_elementwise_dag_one_kernel(cuda_device):
    c = configs.CONFIGS["c2"]
    ops = c.build(**c.small)
    res = run(ops)
    assert len(res.groups) == 1 and res.groups[0].strategy is FusionStrategy.ELEMENTWISE_DAG
    _check_all_outputs("c2", ops, res.env, matmul=False, tol_abs=5e-7)


def test_c2_reference_plan_three_kernels(cuda_device):
    c = configs.CONFIGS["c2"]
    ops = c.build(**c.small)
    res = run(ops, b200=False)
    assert len(res.groups) == 3
    _check_all_outputs("c2", ops, res.env, matmul=False, tol_abs=5e-7)


def test_exact_chain_bitwise(cuda_device):
    """add / mul / max / select chain: bit-identical to IEEE fp32 on the host."""
    r = np.random.default_rng(3)
    M, N = 300, 520
    x, y, z = (r.uniform(-4, 4, (M, N)).astype(np.float32) for _ in range(3))
    from metellus_b200 import Operations

    ops = Operations()
    ops.from_numpy(x, "x")
    ops.from_numpy(y, "y")
    ops.from_numpy(z, "z")
    ops.elementwise("mul", out="a", operands=("x", "y"))
    ops.elementwise("add", out="b", operands=("a", "z"))
    ops.elementwise("mul", out="c", operands=("x", 0.25))
    ops.elementwise("max", out="d", operands=("b", "c"))
    ops.elementwise("gt", out="g", operands=("z", 0.0))
    ops.elementwise("where", out="w", operands=("d", "x", "g"))
    ops.elementwise("subtract", out="o", operands=("w", "z"))
    res = run(ops)
    ref = evaluate(ops, np.float32)
    np.testing.assert_array_equal(res.env["o"], ref["o"])


@pytest.mark.parametrize("K", [4096, 1000, 37])
def test_c3_row_softmax_one_kernel(cuda_device, K):
    X = np.random.default_rng(1).normal(0, 2, (257, K)).astype(np.float32)
    ops = configs.row_softmax(X=X)
    res = run(ops)
    assert len(res.groups) == 1 and res.groups[0].strategy is FusionStrategy.ROW_RESIDENT
    r64 = evaluate(ops, np.float64)
    assert_elementwise_close(res.env["probs"], r64["probs"], rel=2e-6, abs_=1e-9, what="softmax")
    assert_elementwise_close(res.env["row_max_1d"], r64["row_max_1d"], rel=0, abs_=0, what="row max")
    assert_elementwise_close(res.env["row_sum_1d"], r64["row_sum_1d"], rel=2e-6, abs_=0, what="row sum")


def test_c3_reference_plan(cuda_device):
    X = np.random.default_rng(2).normal(0, 2, (128, 512)).astype(np.float32)
    ops = configs.row_softmax(X=X)
    res = run(ops, b200=False)
    assert len(res.groups) == 4
    r64 = evaluate(ops, np.float64)
    assert_elementwise_close(res.env["probs"], r64["probs"], rel=2e-6, abs_=1e-9, what="softmax ref plan")


def test_c3_tensor_sum(cuda_device):
    c = configs.CONFIGS["c3sum"]
    ops = c.build(**c.small)
    res = run(ops)
    r64 = evaluate(ops, np.float64)
    got = float(res.env["total"][0])
    scale = float(np.abs(ops.uploads["X"]).astype(np.float64).sum())
    assert abs(got - r64["total"][0]) <= 1e-6 * scale


def test_c1_matmul_bias_relu(cuda_device):
    c = configs.CONFIGS["c1"]
    ops = c.build(**c.small)
    res = run(ops)
    assert len(res.groups) == 1
    _check_all_outputs("c1", ops, res.env, matmul=True)


def test_c4_attention_small(cuda_device):
    c = configs.CONFIGS["c4"]
    ops = c.build(**c.small)
    res = run(ops)
    r64 = evaluate(ops, np.float64)
    r32 = evaluate(ops, np.float32)
    assert_matmul_close(res.env["O"], r64["O"], r32["O"], what="attention")


def test_c5_mlp_small(cuda_device):
    c = configs.CONFIGS["c5"]
    ops = c.build(**c.small)
    res = run(ops)
    r64 = evaluate(ops, np.float64)
    r32 = evaluate(ops, np.float32)
    assert_matmul_close(res.env["out"], r64["out"], r32["out"], what="mlp")
