"""The allocation-free reduction entry point, ``mt_reduce_rows_noalloc``.

Some callers cannot allocate device memory — code that runs inside another
framework's device-memory budget (a serving process whose caching allocator already
owns the GPU) or a latency-critical loop that must not allocate. For them the C ABI
offers this variant of ``mt_reduce_rows``: same kernel, but its scratch is a fixed
256 KiB array inside the library instead of pool memory.

This file is named so pytest collects it last. The test calls the entry point
through the C ABI on caller-owned device pointers, twice in a row (the shared array
keeps the previous call's contents), and requires each result to equal the allocating
entry point's bit for bit (same kernel, same plan, deterministic combine order) and to
agree with the fp64 sum / max of the input (|err| <= 1e-6 * sum|x| for sums, exact for
max). One case passes a stream the caller created (torch) on torch-owned tensors. It
also checks that oversized requests are rejected."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from metellus_b200.runtime import backend
from metellus_b200.runtime.buffer import Buffer

pytestmark = pytest.mark.gpu


def _noalloc(dev, in_ptr, out_ptr, rows, cols, ld, op, stream=None):
    rc = backend.lib().mt_reduce_rows_noalloc(dev, ctypes.c_void_p(in_ptr), ctypes.c_void_p(out_ptr), rows,
                                              cols, ld, backend.REDUCE_OPS[op],
                                              None if stream is None else ctypes.c_void_p(stream))
    backend._check(rc)


def _check_fp64(X, got, op):
    x64 = X.astype(np.float64)
    if op == "max":
        np.testing.assert_array_equal(got, X.max(axis=1))
    else:
        ref = x64.sum(axis=1)
        scale = np.abs(x64).sum(axis=1)
        assert np.all(np.abs(got - ref) <= 1e-6 * scale), (got, ref)


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
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32), err_msg=f"call {call}")
        _check_fp64(X, got, op)


def test_noalloc_on_a_caller_stream(cuda_device):
    """A host framework passes its own stream and its own device tensors."""
    import torch

    dev = backend.current_device()
    rows, cols = 2, 1 << 20
    X = np.random.default_rng(12).normal(0, 1, (rows, cols)).astype(np.float32)
    s = torch.cuda.Stream(device=dev)
    tx = torch.from_numpy(X).to(f"cuda:{dev}")
    outs = []
    for _ in range(2):
        to = torch.full((rows,), float("nan"), device=f"cuda:{dev}")
        s.wait_stream(torch.cuda.current_stream(dev))
        _noalloc(dev, tx.data_ptr(), to.data_ptr(), rows, cols, cols, "sum", stream=s.cuda_stream)
        s.synchronize()
        outs.append(to.cpu().numpy())
    assert torch.cuda.current_device() == dev
    np.testing.assert_array_equal(outs[0], outs[1])
    bx = Buffer.from_numpy(X)
    ref_out = Buffer.zeros(4 * rows)
    backend.reduce_rows(bx.handle, ref_out.handle, rows, cols, cols, "sum")
    np.testing.assert_array_equal(outs[0], ref_out.numpy((rows,)))
    _check_fp64(X, outs[0], "sum")


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
