"""The allocation-free reduction entry point, ``mt_reduce_rows_noalloc``.

Some callers cannot allocate device memory — code that runs inside another
framework's device-memory budget (a serving process whose caching allocator already
owns the GPU) or a latency-critical loop that must not allocate. For them the C ABI
offers this variant of ``mt_reduce_rows``: same kernel, but its scratch is a fixed
256 KiB array inside the library instead of pool memory.

This file is named so pytest collects it last. The test calls the entry point
through the C ABI on caller-owned device pointers, twice in a row (the shared array
keeps the previous call's contents), and compares each result with the allocating
entry point's within the reduction tolerance used by tests/test_gpu_reduce.py
(one ulp of the result). It also checks that oversized requests are rejected."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from metellus_b200.runtime import backend
from metellus_b200.runtime.buffer import Buffer

pytestmark = pytest.mark.gpu


def _noalloc(dev, in_ptr, out_ptr, rows, cols, ld, op):
    rc = backend.lib().mt_reduce_rows_noalloc(dev, ctypes.c_void_p(in_ptr), ctypes.c_void_p(out_ptr), rows,
                                              cols, ld, backend.REDUCE_OPS[op], None)
    backend._check(rc)


@pytest.mark.parametrize("op,shape", [("sum", (1, 1 << 22)), ("max", (3, 300_001)), ("sum", (64, 70_000))])
def test_noalloc_matches_allocating_entry(cuda_device, op, shape):
    rows, cols = shape
    r = np.random.default_rng(11)
    dev = backend.current_device()
    for call in range(2):
        X = r.normal(0, 2, shape).astype(np.float32)
        bx = Buffer.from_numpy(X)
        ref_out, got_out = Buffer.zeros(4 * rows), Buffer.zeros(4 * rows)
        backend.reduce_rows(bx.handle, ref_out.handle, rows, cols, cols, op)
        _noalloc(dev, backend.buffer_ptr(bx.handle), backend.buffer_ptr(got_out.handle), rows, cols, cols, op)
        want = ref_out.numpy((rows,))
        got = got_out.numpy((rows,))
        ulp = np.spacing(np.abs(want))
        assert np.all(np.abs(got - want) <= ulp), (call, got, want)


def test_noalloc_rejects_too_many_rows(cuda_device):
    dev = backend.current_device()
    rows, cols = 70_000, 8
    bx, bo = Buffer.zeros(4 * rows * cols), Buffer.zeros(4 * rows)
    with pytest.raises(RuntimeError, match="exceed 65535"):
        _noalloc(dev, backend.buffer_ptr(bx.handle), backend.buffer_ptr(bo.handle), rows, cols, cols, "sum")


def test_noalloc_rejects_scratch_overflow(cuda_device):
    """40,000 one-split rows need 40,000 x (8 + 4) B = 480 KB of scratch, more than
    the 256 KiB array: rejected with a message naming the limit, before any launch
    (the buffers are still sized for the request)."""
    dev = backend.current_device()
    rows, cols = 40_000, 8
    bx, bo = Buffer.zeros(4 * rows * cols), Buffer.zeros(4 * rows)
    with pytest.raises(RuntimeError, match="bytes of scratch"):
        _noalloc(dev, backend.buffer_ptr(bx.handle), backend.buffer_ptr(bo.handle), rows, cols, cols, "sum")
