"""Schedule KernelGroups into a Runtime (reference: src/orchestrator/scheduler.py:59-221).

Same plan: validate that uploads cover exactly the external input buffers; upload
inputs; allocate every other bound buffer in first-use order; prime (compile) each
kernel; dispatch in order; after the dispatch that last uses a buffer, download every
declared tensor backed by it (views gathered through their strides, the owner last)
and free it. Fused-away intermediates are never bound, so never allocated or
returned.

On CUDA the dispatches are asynchronous and stream ordered; frees are stream ordered
too (cudaFreeAsync), so "free at last use" never waits for the device — only the
downloads do.
"""

from __future__ import annotations

import numpy as np

from metellus_b200.orchestrator.builder import Operations
from metellus_b200.orchestrator.dag import build_dag
from metellus_b200.orchestrator.kernel_group import STATUS_KEY, KernelGroup
from metellus_b200.runtime.program import (
    Allocate,
    CheckStatus,
    Fill,
    Dispatch,
    Download,
    Free,
    FromNumpy,
    Runtime,
    RuntimeFragment,
)


def dispatch_of(g: KernelGroup, time_key: str | None = None) -> Dispatch:
    """Launch step of a group: parameters are its bindings then its scratch buffers."""
    keys = tuple(g.bindings) + tuple(k for k, _ in g.scratch)
    return Dispatch(kernel=g.kernel, bindings=keys, dims=g.dims, grid=g.grid, threads=g.threads,
                    time_key=time_key, tmaps=g.tmaps, cluster_x=g.cluster_x or 1)


def scratch_of(groups: tuple[KernelGroup, ...]) -> dict[str, int]:
    out: dict[str, int] = {}
    for g in groups:
        for k, n in g.scratch:
            out[k] = max(out.get(k, 0), n)
    return out


def buffer_sizes(ops: Operations, groups: tuple[KernelGroup, ...]) -> dict[str, int]:
    """Bytes of every buffer key the plan touches."""
    tensors = ops.tensors
    sizes: dict[str, int] = {}
    for op in ops.build():
        sizes[op.out.buffer_key] = op.out.nbytes
    for name in ops.uploads:
        sizes[tensors[name].buffer_key] = tensors[name].nbytes
    for g in groups:
        for key, nbytes in g.scratch:
            sizes[key] = max(sizes.get(key, 0), nbytes)
    return sizes


def schedule(ops: Operations, groups: tuple[KernelGroup, ...], *, profile: bool = False) -> Runtime:
    program = ops.build()
    dag = build_dag(program)
    tensors = ops.tensors
    uploads = ops.uploads

    produced_keys = {op.out.buffer_key for op in program}
    required: set[str] = set()
    for n in dag.inputs:
        bk = tensors[n].buffer_key
        if bk not in produced_keys:
            required.add(bk)
    provided = set(uploads)
    missing, extra = required - provided, provided - required
    if missing:
        raise ValueError(f"schedule: input buffers {sorted(missing)} have no from_numpy upload")
    if extra:
        raise ValueError(f"schedule: uploads {sorted(extra)} do not correspond to any program input")

    nbytes = buffer_sizes(ops, groups)
    input_keys = {tensors[n].buffer_key for n in uploads}
    materialized = set(input_keys)
    for g in groups:
        materialized.update(g.bindings)
    names_per_key: dict[str, list[str]] = {}
    for name, t in tensors.items():
        if name in uploads or t.buffer_key not in materialized:
            continue
        names_per_key.setdefault(t.buffer_key, []).append(name)

    last_use: dict[str, int] = {}
    for i, g in enumerate(groups):
        for k in g.bindings:
            last_use[k] = i

    steps: list[RuntimeFragment] = []
    for name, arr in uploads.items():
        steps.append(FromNumpy(name=tensors[name].buffer_key, source=arr))
    scratch = scratch_of(groups)
    for k, n in scratch.items():
        steps.append(Allocate(name=k, nbytes=n))
        steps.append(Fill(name=k, byte_value=0))
    seen = set(input_keys)
    for g in groups:
        for k in g.bindings:
            if k not in seen:
                steps.append(Allocate(name=k, nbytes=nbytes[k]))
                seen.add(k)
        steps.append(g.kernel)
    freed: set[str] = set()
    for i, g in enumerate(groups):
        steps.append(dispatch_of(g, f"t_{i}" if profile else None))
        for k in dict.fromkeys(g.bindings):
            if k in freed or last_use.get(k) != i:
                continue
            names = names_per_key.get(k, ())
            for vn in (n for n in names if n != k):
                t = tensors[vn]
                steps.append(Download(name=t.buffer_key, shape=t.shape, dtype=np.float32, into=t.name,
                                      row_stride=t.row_stride, col_stride=t.col_stride,
                                      batch_stride=t.batch_stride))
            if k in names:
                t = tensors[k]
                steps.append(Download(name=k, shape=t.shape, dtype=np.float32, into=t.name))
            else:
                steps.append(Free(name=k))
            freed.add(k)
    for k in scratch:
        if k == STATUS_KEY:
            steps.append(CheckStatus(name=k))
        steps.append(Free(name=k))
    return Runtime(tuple(steps))
