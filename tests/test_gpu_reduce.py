"""GPU parity of the native split-row reduction (``mt_reduce_rows``): whole-tensor
and few-long-row reductions through the public API and through the C ABI, every op,
against the fp64 oracle. Sum / product accumulate in fp64, so the result is the
fp64 value rounded once: |gpu - fp64| <= 1 ulp of the result (plus 1e-7 of sum|x| for
cancelling sums)."""

from __future__ import annotations

import numpy as np
import pytest

from metellus_b200 import Operations, configs, run
from metellus_b200.runtime import backend
from metellus_b200.runtime.buffer import Buffer
from oracle.ir_eval import evaluate

pytestmark = pytest.mark.gpu


def _close(got, ref64, x):
    ref32 = np.float32(ref64)
    ulp = np.spacing(np.abs(ref32)).astype(np.float64)
    scale = 1e-7 * np.abs(x.astype(np.float64)).sum(axis=-1)
    assert np.all(np.abs(got.astype(np.float64) - ref64) <= ulp + scale), (got, ref64)


@pytest.mark.parametrize("op", ["sum", "max", "min", "product"])
@pytest.mark.parametrize("shape", [(1, 1 << 20), (3, 200_003), (7, 65_536)])
def test_split_reduction_api(cuda_device, op, shape):
    r = np.random.default_rng(7)
    M, K = shape
    X = (1.0 + r.uniform(-1e-4, 1e-4, shape)).astype(np.float32) if op == "product" else \
        r.normal(0, 2, shape).astype(np.float32)
    ops = Operations()
    ops.from_numpy(X, "X")
    ops.reduction(op, out="R", x="X", axis=-1)
    res = run(ops)
    assert res.groups[0].pipe == "native"
    ref = evaluate(ops, np.float64)["R"]
    _close(res.env["R"], ref, X)


def test_whole_tensor_sum_config(cuda_device):
    c = configs.CONFIGS["c3sum"]
    ops = c.build(M=1024, K=4096)
    res = run(ops)
    ref = evaluate(ops, np.float64)["total"]
    _close(res.env["total"], ref, ops.uploads["X"].reshape(1, -1))


def test_reduce_rows_c_abi_repeated(cuda_device):
    """Direct C-ABI call, twice in a row on the same buffers (scratch tickets reset)."""
    r = np.random.default_rng(9)
    X = r.normal(0, 1, (2, 300_000)).astype(np.float32)
    bx, bo = Buffer.from_numpy(X), Buffer.zeros(8)
    for _ in range(2):
        backend.reduce_rows(bx.handle, bo.handle, 2, 300_000, 300_000, "sum")
        got = bo.numpy((2,))
        _close(got, X.astype(np.float64).sum(axis=1), X)


def test_reduce_rows_rejects_bad_sizes(cuda_device):
    bx, bo = Buffer.zeros(16), Buffer.zeros(4)
    with pytest.raises(RuntimeError, match="too small"):
        backend.reduce_rows(bx.handle, bo.handle, 1, 1000, 1000, "sum")
    with pytest.raises(RuntimeError, match="empty"):
        backend.reduce_rows(bx.handle, bo.handle, 0, 4, 4, "sum")
