"""GPU parity of ``Executable`` (compile once, persistent buffers, CUDA-graph replay)
against ``run`` on the same program: repeated calls with new inputs, the graph
captured on the second call. Covers every pipe: elementwise DAG, row-resident,
native split reduction, tcgen05 GEMM and attention."""

from __future__ import annotations

import numpy as np
import pytest

from metellus_b200 import Executable, configs, run
from metellus_b200.runtime import backend

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("key", ["c1", "c2", "c3", "c3sum", "c4", "c5"])
def test_executable_matches_run(cuda_device, key):
    c = configs.CONFIGS[key]
    exe = None
    try:
        for seed in range(3):
            ops = c.build(**c.small, seed=seed)
            if exe is None:
                exe = Executable(ops, outputs=(c.output,))
            want = run(ops).env[c.output]
            got = exe(ops.uploads)[c.output]
            np.testing.assert_array_equal(got.reshape(want.shape), want)
        assert exe._graph is not None  # replayed from the captured graph
    finally:
        if exe is not None:
            exe.close()


def test_executable_pinned_async(cuda_device):
    c = configs.CONFIGS["c2"]
    ops = c.build(**c.small, seed=5)
    exe = Executable(ops, outputs=("out",))
    pins = {}
    for n, a in ops.uploads.items():
        p = backend.PinnedArray(a.shape)
        p.array[...] = a
        pins[n] = p
    out = backend.PinnedArray(ops.tensors["out"].shape)
    for _ in range(3):
        exe({n: p.array for n, p in pins.items()}, out={"out": out.array}, wait=False)
    exe.synchronize()
    np.testing.assert_array_equal(out.array, run(ops).env["out"])
    exe.close()


def test_executable_rejects_unknown_input(cuda_device):
    c = configs.CONFIGS["c2"]
    ops = c.build(**c.small)
    exe = Executable(ops)
    with pytest.raises(KeyError):
        exe({"nope": np.zeros(3, np.float32)})
    exe.close()
