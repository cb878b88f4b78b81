"""GPU parity of the fused attention kernels against the fp64 oracle: the tcgen05
3xTF32 flash kernel (head dim 64, whole 64-key blocks; ragged query tiles included)
and the FFMA kernel it falls back to for other shapes. The output and the exposed
row statistics (max of the scaled scores, sum of exponentials) are checked."""

from __future__ import annotations

import numpy as np
import pytest

from metellus_b200 import configs, run
from oracle.ir_eval import evaluate
from tests.tolerances import assert_matmul_close

pytestmark = pytest.mark.gpu


def _check(ops, res):
    r64 = evaluate(ops, np.float64)
    r32 = evaluate(ops, np.float32)
    assert_matmul_close(res.env["O"], r64["O"], r32["O"], what="attention O")
    # the row statistics come out of the Q K^T product: matmul tolerance (normwise)
    for stat in ("row_max_1d", "row_sum_1d"):
        if stat in res.env:
            assert_matmul_close(res.env[stat], r64[stat], r32[stat], what=stat)


@pytest.mark.parametrize("B,S", [(2, 128), (3, 320), (1, 1024), (4, 64)])
def test_tc_attention(cuda_device, B, S):
    ops = configs.CONFIGS["c4"].build(B=B, S=S, D=64, seed=B * 1000 + S)
    res = run(ops)
    assert [g.pipe for g in res.groups] == ["tcgen05"]
    _check(ops, res)


@pytest.mark.parametrize("B,S,D", [(2, 200, 64), (2, 128, 128)])
def test_ffma_attention_fallback(cuda_device, B, S, D):
    ops = configs.CONFIGS["c4"].build(B=B, S=S, D=D, seed=7)
    res = run(ops)
    assert [g.pipe for g in res.groups] == ["ffma"]
    _check(ops, res)
