"""Strong-scaling shards of the benchmark configurations (``configs.shard``): each
rank's rows / heads are a contiguous block of the one full configuration, the blocks
cover it exactly, and replicated operands (C5's weights) are identical on every rank."""

from __future__ import annotations

import numpy as np
import pytest

from metellus_b200 import configs
from metellus_b200.orchestrator.assembly.tc_matmul import _pair_group_m

SMALL = {"c2": dict(M=64, N=32), "c3": dict(M=64, K=32), "c3sum": dict(M=64, K=32),
         "c4": dict(B=8, S=64, D=64), "c5": dict(M=64, D=32, F=64)}
ROWS = {"c2": ("x", 0), "c3": ("X", 0), "c3sum": ("X", 0), "c4": ("Q", 0), "c5": ("X", 0)}


@pytest.mark.parametrize("key", sorted(SMALL))
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_shards_tile_the_full_configuration(key, world):
    full = configs.CONFIGS[key].build(**SMALL[key]).uploads
    name, _ = ROWS[key]
    parts = []
    for rank in range(world):
        ops, shape = configs.shard(key, world, rank, **SMALL[key])
        arr = ops.uploads[name]
        axis = configs.SHARD_AXIS[key]
        assert arr.shape[0] == shape[axis]
        parts.append(arr)
        if key == "c5":
            for w in ("W1", "W3", "W2", "b1", "b2"):
                np.testing.assert_array_equal(ops.uploads[w], full[w])
    np.testing.assert_array_equal(np.concatenate(parts), full[name])


def test_c1_ranks_are_replicas():
    a, _ = configs.shard("c1", 4, 0, M=64, K=32, N=48)
    b, _ = configs.shard("c1", 4, 3, M=64, K=32, N=48)
    for n in ("A", "B", "bias"):
        np.testing.assert_array_equal(a.uploads[n], b.uploads[n])


def test_pair_group_sizes_follow_the_measured_choice():
    assert _pair_group_m(2048) == 16     # C5 dual GEMM
    assert _pair_group_m(8192) == 2      # C5 down-projection
