"""Regenerate ``pipe_table.json``: device time of every matmul variant on a grid of
shapes, measured on the GPU this runs on (a B200).

    python -m metellus_b200.orchestrator.assembly.measure_pipe_table [--out PATH]

For each shape (M, N, K, anchors) it plans the program under each forced variant
(``pipe_table.forced``: the SIMT FFMA tile, and the tcgen05 kernel as CTA pairs, one
CTA, or split-K pairs), checks that the plan really uses that variant, and times the
whole program (one kernel on the tensor-core pipe; the FFMA plan of the diamond may
take more) with CUDA events (median of 7 launches after 2 warm-ups; operands
resident, warm L2 — the same conditions for every variant). One anchor is ``C = A @
B``; two anchors are the shared-input diamond ``U = (H @ W1) * (H @ W3)``. The fastest
variant is the shape's pick.
"""

from __future__ import annotations

import argparse
import json
import statistics
import time

import numpy as np

from metellus_b200.orchestrator.assembly import pipe_table

SHAPES_1 = [
    (128, 128, 128), (256, 256, 256), (512, 512, 512), (1024, 1024, 1024), (2048, 2048, 2048),
    (4096, 4096, 4096), (8192, 8192, 8192),
    (1024, 1024, 64), (1024, 64, 1024),          # per-head attention products (C4)
    (16384, 2048, 8192),                         # C5 down-projection
    (4096, 256, 4096), (256, 4096, 4096), (512, 512, 8192), (8192, 8192, 256), (2048, 2048, 256),
    (256, 320, 192),                             # C1's test-size shape
]
SHAPES_2 = [
    (16384, 8192, 2048),                         # C5 up-projections (dual GEMM)
    (4096, 4096, 4096), (1024, 1024, 1024), (2048, 2048, 512), (256, 512, 256),
]


def _program(M: int, N: int, K: int, nb: int, rng):
    from metellus_b200 import Operations

    ops = Operations()
    if nb == 1:
        ops.from_numpy(rng.normal(size=(M, K)).astype(np.float32), "A")
        ops.from_numpy(rng.normal(size=(K, N)).astype(np.float32), "B")
        ops.matmul("A", "B", "C")
    else:
        ops.from_numpy(rng.normal(size=(M, K)).astype(np.float32), "H")
        ops.from_numpy(rng.normal(size=(K, N)).astype(np.float32), "W1")
        ops.from_numpy(rng.normal(size=(K, N)).astype(np.float32), "W3")
        ops.matmul("H", "W1", "z1")
        ops.matmul("H", "W3", "z3")
        ops.elementwise("mul", out="U", operands=("z1", "z3"))
    return ops


def _variant_of(g) -> str:
    if g.pipe != "tcgen05":
        return "ffma"
    frag = g.kernel.fragments[0]
    if getattr(frag, "pair", None) is not None:
        return "pair"
    return "splitk" if getattr(frag, "splitk", 1) > 1 else "one"


def time_variant(M: int, N: int, K: int, nb: int, variant: str, rng) -> float | None:
    from metellus_b200.api.run import compile_program
    from metellus_b200.orchestrator.scheduler import buffer_sizes, dispatch_of, scratch_of
    from metellus_b200.runtime import backend
    from metellus_b200.runtime.buffer import Buffer

    ops = _program(M, N, K, nb, rng)
    with pipe_table.forced(variant):
        groups = compile_program(ops)
    mm = [g for g in groups if any(type(o).__name__ == "MatmulOp" for o in g.ops)]
    if not mm or any(_variant_of(g) != variant for g in mm):
        return None
    env = {}
    tensors = ops.tensors
    for name, arr in ops.uploads.items():
        env[tensors[name].buffer_key] = Buffer.from_numpy(arr)
    for k, n in scratch_of(groups).items():
        env[k] = Buffer.zeros(n)
    sizes = buffer_sizes(ops, groups)
    dispatches = [dispatch_of(g) for g in groups]
    for d in dispatches:
        for k in d.bindings:
            if k not in env:
                env[k] = Buffer.zeros(sizes[k])
    ts = []
    for i in range(9):
        e0, e1 = backend.Event(), backend.Event()
        e0.record()
        for d in dispatches:
            d.execute(env)
        e1.record()
        backend.sync()
        if i >= 2:
            ts.append(e0.elapsed_ms(e1) * 1e3)
    for b in env.values():
        b.release()
    return statistics.median(ts)


def _device_name() -> str:
    import torch

    return torch.cuda.get_device_name(0) if torch.cuda.is_available() else "unknown"


def main() -> None:
    from metellus_b200.runtime import backend

    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(pipe_table.TABLE_PATH))
    args = ap.parse_args()
    backend.init()
    rng = np.random.default_rng(0)
    out = []
    for nb, shapes in ((1, SHAPES_1), (2, SHAPES_2)):
        for M, N, K in shapes:
            us = {}
            for v in pipe_table.VARIANTS:
                if v == "splitk" and nb == 2:
                    continue
                t = time_variant(M, N, K, nb, v, rng)
                if t is not None:
                    us[v] = round(t, 2)
            best = min(us, key=us.get)
            out.append({"shape": [M, N, K, nb], "us": us, "best": best})
            print(json.dumps(out[-1]), flush=True)
    doc = {
        "_about": "device time (us, median of 7 warm launches, CUDA events) of each matmul variant; "
                  "'best' is the pick. Regenerate: python -m metellus_b200.orchestrator.assembly.measure_pipe_table",
        "device": _device_name(),
        "when": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime()),
        "entries": out,
    }
    with open(args.out, "w") as f:
        json.dump(doc, f, indent=1)
        f.write("\n")


if __name__ == "__main__":
    main()
