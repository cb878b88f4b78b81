"""GPU runs of the strided-copy (ShapeOp) kernel for reshapes that cannot be views:
the reference's end-to-end shape cases (a transpose followed by a flatten or a 2-D
reshape, a tail that does not fill a block, several blocks), bit-exact against numpy."""

from __future__ import annotations

import numpy as np
import pytest

from metellus_b200 import Operations, run
from metellus_b200.orchestrator.kernel_group import FusionStrategy

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape,new_shape,seed", [((8, 16), (128,), 0), ((8, 16), (32, 4), 1), ((10, 13), (130,), 2),
                                                  ((32, 32), (1024,), 3), ((300, 70), (140, 150), 4)])
def test_transpose_then_reshape(cuda_device, shape, new_shape, seed):
    x = np.random.default_rng(seed).standard_normal(shape).astype(np.float32)
    ops = Operations()
    ops.from_numpy(x, "X")
    ops.transpose("X", out="Xt")
    ops.reshape("Xt", new_shape, out="Y")
    res = run(ops)
    assert [g.strategy for g in res.groups] == [FusionStrategy.STANDALONE_SHAPE]
    np.testing.assert_array_equal(res.env["Y"], x.T.reshape(new_shape))
