"""Benchmark of the Metellus B200 backend on the BASELINE configurations.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2] [--impl ours|reference]

One step = one run of the whole fused program over one batch of synthetic inputs
(seeded, the configuration's shapes and distributions). Default workload: config C2
(the elementwise DAG, x/y/z fp32 8192x8192), the configuration the metric is quoted
on that fits one GPU; ``--config c1|c3|c3sum|c4|c5`` runs the others.

Multi-GPU (torchrun, one process per GPU): every rank runs the same per-GPU shard of
a row-/batch-sharded problem (weak scaling; no data-path collective), timing is the
max over ranks of CUDA-event device time, ``value`` = work of all ranks / that time.

Printed JSON keys: the driver contract (metric, value, unit, n_gpus, steps, warmup,
ms_per_step, higher_is_better, scaling, vs_baseline, dtype, data, config) plus
``e2e`` (same metric through the public API with pinned host inputs, H2D + D2H
inside the timed region), ``roofline`` (dominant kernel vs MEASURED_PEAKS.json),
``cpu_baseline`` (the CPU oracle on a bounded sample, rank 0, N=1), ``clocks``
(nvidia-smi samples during the timed region) and ``gpu_launches``.

``--impl reference`` times the reference's CPU path for this program (the numpy
restatement in oracle/, all host threads; MLX-CPU is not installable here) on a
bounded sample and prints the same metric.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from metellus_b200 import configs  # noqa: E402

L2_BYTES = 126 * 1024 * 1024


def parse() -> argparse.Namespace:
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--config", default="c2", choices=sorted(configs.CONFIGS))
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu", action="store_true")
    p.add_argument("--profile", action="store_true",
                   help="profiling capture mode: no clock soak, no e2e, no CPU baseline")
    p.add_argument("--shape", default="", help="override the per-GPU shape, e.g. M=2048,N=8192 "
                   "(profiling captures on a smaller case)")
    return p.parse_args()


def shard_shape(key: str) -> dict:
    """Per-GPU shape: the full single-GPU configuration (weak scaling)."""
    return dict(configs.CONFIGS[key].full)


def metric_of(key: str) -> tuple[str, str, bool]:
    bound = configs.CONFIGS[key].bound
    if bound == "hbm":
        return "fused-program GB/s (% HBM roofline)", "GB/s", True
    return "fused-program TFLOP/s (% roofline)", "TFLOP/s", True


def amount(key: str, shape: dict) -> float:
    flops, nbytes = configs.algorithmic_work(key, **shape)
    return nbytes / 1e9 if configs.CONFIGS[key].bound == "hbm" else flops / 1e12


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d.get("hbm_gbs", 6650.0), "src": "measured", **d}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


class ClockSampler:
    """nvidia-smi SM clock / throttle sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int) -> None:
        self.index = index
        self.proc = None
        self.path = Path(tempfile.mkstemp(suffix=".csv")[1])

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in self.path.read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9:
                rows.append(f)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        sm = []
        smax = None
        for f in rows:
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                pass
            for i, n in enumerate(names):
                if f[5 + i].lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# -- CPU baseline / reference arm -------------------------------------------------------


def cpu_sample_shape(key: str, frac_rows: int) -> dict:
    s = dict(configs.CONFIGS[key].full)
    if key in ("c2",):
        s["M"] = max(1, s["M"] // frac_rows)
    elif key in ("c3", "c3sum"):
        s["M"] = max(1, s["M"] // frac_rows)
    elif key == "c4":
        s["B"] = max(1, s["B"] // frac_rows)
    elif key == "c5":
        s["M"] = max(16, s["M"] // frac_rows)
    return s


def time_cpu(key: str, threads: int, frac_rows: int, reps: int = 1) -> tuple[float, dict, int]:
    """Time the oracle's fp32 evaluation of a row/batch sample split over ``threads``
    host threads (numpy releases the GIL in its kernels). Returns (seconds per sample,
    sample shape, threads used)."""
    from oracle.ir_eval import evaluate

    shape = cpu_sample_shape(key, frac_rows)
    c = configs.CONFIGS[key]
    # split the sample into `threads` row shards, each an independent program
    parts = []
    split_key = {"c4": "B"}.get(key, "M")
    total = shape[split_key]
    n = max(1, min(threads, total))
    base = total // n
    for i in range(n):
        s = dict(shape)
        s[split_key] = base + (1 if i < total - base * n else 0)
        if s[split_key] > 0:
            parts.append(c.build(**s, seed=i))
    best = math.inf
    with ThreadPoolExecutor(max_workers=len(parts)) as ex:
        for _ in range(reps):
            t0 = time.perf_counter()
            list(ex.map(lambda o: evaluate(o, np.float32), parts))
            best = min(best, time.perf_counter() - t0)
    return best, shape, len(parts)


def reference_arm(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    key = args.config
    metric, unit, hib = metric_of(key)
    threads = os.cpu_count() or 1
    frac = {"c2": 32, "c3": 32, "c3sum": 32, "c4": 32, "c5": 256, "c1": 1}[key]
    for _ in range(args.warmup):
        time_cpu(key, threads, frac * 4)
    times = []
    shape = None
    used = 1
    for _ in range(args.steps):
        t, shape, used = time_cpu(key, threads, frac)
        times.append(t)
    sec = statistics.median(times)
    value = amount(key, shape) / sec
    line = {
        "impl": "reference", "metric": metric, "value": value, "unit": unit, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": hib,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
        "config": {"workload": key, **shape, "full": configs.CONFIGS[key].full},
        "cpu_baseline": {"value": value, "unit": unit, "cores": used, "kind": "port",
                         "sample": f"{shape} per step (1/{frac} of the configuration), numpy fp32 "
                                   f"restatement of the reference program, {used} host threads"},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# -- GPU arm --------------------------------------------------------------------------------


def main() -> None:
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import torch
        import torch.distributed as tdist

        torch.cuda.set_device(local)
        tdist.init_process_group("nccl", device_id=torch.device("cuda", local))
        dist = tdist

    from metellus_b200 import distributed
    from metellus_b200.api.run import compile_program
    from metellus_b200.orchestrator.scheduler import buffer_sizes, dispatch_of
    from metellus_b200.runtime import backend
    from metellus_b200.runtime.buffer import Buffer

    def trace(msg: str) -> None:
        if os.environ.get("METELLUS_TRACE"):
            print(f"[rank {rank}] {msg}", file=sys.stderr, flush=True)

    key = args.config
    # binds the GPU; for N > 1 and a combined reduction also creates the NCCL communicator
    distributed.init(nccl=key == "c3sum")
    trace("device and communicator ready")
    shape = shard_shape(key)
    for kv in filter(None, args.shape.split(",")):
        k, v = kv.split("=")
        shape[k] = int(v)
    ops = configs.CONFIGS[key].build(**shape, seed=rank)
    # the whole-tensor sum of a row-sharded X: local fp64 partial + NCCL all-reduce
    combine = (configs.CONFIGS[key].output,) if key == "c3sum" and world > 1 else ()
    with distributed.combining(*combine):
        groups = compile_program(ops)
    for g in groups:
        _ = g.kernel.handle  # compile before timing
    tensors = ops.tensors
    uploads = ops.uploads
    sizes = buffer_sizes(ops, groups)
    env = {}
    for name, arr in uploads.items():
        env[tensors[name].buffer_key] = Buffer.from_numpy(arr)
    dispatches = [dispatch_of(g) for g in groups]
    for d in dispatches:
        for k in d.bindings:
            if k not in env:
                env[k] = Buffer.zeros(sizes[k])
    in_bytes = sum(a.nbytes for a in uploads.values())
    needs_flush = in_bytes < 2 * L2_BYTES
    flush = Buffer(256 * 1024 * 1024) if needs_flush else None

    def step() -> None:
        for d in dispatches:
            d.execute(env)

    def barrier() -> None:
        backend.sync()
        if dist is not None:
            dist.barrier()

    trace("compiled and allocated")
    for _ in range(max(args.warmup, 3)):
        step()
    barrier()
    trace("warm-up done")
    # Timed steps replay the dispatch list from a CUDA graph (captured after the
    # warm-up has loaded every module), so a step is one graph launch and the host
    # stays ahead of the device; per-kernel times come from a second, per-dispatch pass.
    # Programs with an NCCL combine run their dispatches directly.
    graph = None
    if not any("nccl" in (g.pipe or "") for g in groups):
        backend.graph_begin()
        try:
            step()
        finally:
            graph = backend.graph_end()
        backend.graph_launch(graph)
        barrier()

    def timed_step() -> None:
        if graph is not None:
            backend.graph_launch(graph)
        else:
            step()
    ev = [(backend.Event(), backend.Event()) for _ in range(args.steps)]
    gev = [[(backend.Event(), backend.Event()) for _ in groups] for _ in range(args.steps)]
    # Clock sampling covers a ~1 s soak of the same steps right before the timed
    # region and the timed region itself (nvidia-smi samples every 100 ms).
    sampler = ClockSampler(local)
    sampler.start()
    t_soak = time.perf_counter()
    while not args.profile and time.perf_counter() - t_soak < 1.0:
        for _ in range(8):
            timed_step()
        backend.sync()
    barrier()
    # The L2 flush of step i runs after step i's closing event, so the host enqueues
    # step i + 1 while the flush occupies the GPU and no launch gap lands inside a step.
    if flush is not None:
        backend.fill_buffer(flush.handle, 0xFF, wait=False)
    t_wall = time.perf_counter()
    for i in range(args.steps):
        ev[i][0].record()
        timed_step()
        ev[i][1].record()
        if flush is not None:
            backend.fill_buffer(flush.handle, i & 0xFF, wait=False)
    barrier()
    wall = time.perf_counter() - t_wall
    clocks = sampler.stop()
    step_ms = [a.elapsed_ms(b) for a, b in ev]
    # per-kernel device times (same inputs, same flush), for the roofline of the
    # dominant kernel
    if flush is not None:
        backend.fill_buffer(flush.handle, 0xFF, wait=False)
    for i in range(args.steps):
        for j, d in enumerate(dispatches):
            gev[i][j][0].record()
            d.execute(env)
            gev[i][j][1].record()
        if flush is not None:
            backend.fill_buffer(flush.handle, i & 0xFF, wait=False)
    barrier()
    if graph is not None:
        backend.graph_destroy(graph)
    group_ms = [statistics.mean(gev[i][j][0].elapsed_ms(gev[i][j][1]) for i in range(args.steps))
                for j in range(len(groups))]
    ms = statistics.mean(step_ms)
    if dist is not None:
        import torch

        t = torch.tensor([ms], device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())

    per_rank = amount(key, shape)
    value = per_rank * world / (ms / 1e3)
    metric, unit, hib = metric_of(key)

    # dominant kernel roofline
    j = int(np.argmax(group_ms))
    gdom = groups[j]
    pk = peaks()
    flops, nbytes = configs.algorithmic_work(key, **shape)
    if configs.CONFIGS[key].bound == "hbm":
        dom_bytes = kernel_bytes(gdom, ops)
        achieved = dom_bytes / (group_ms[j] / 1e3) / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / pk["hbm_gbs"], "traffic": committed_traffic(key, gdom),
                "kernel": gdom.kernel.function_name, "peak_src": f"{pk['src']} hbm_gbs",
                "algorithmic_bytes": dom_bytes}
    else:
        kflops = kernel_flops(gdom)
        achieved = kflops / (group_ms[j] / 1e3) / 1e12
        pipe_peak, src = tensor_peak(gdom, pk)
        roof = {"bound": "tensor", "achieved": achieved, "peak": pipe_peak, "unit": "TFLOP/s",
                "frac": achieved / pipe_peak, "traffic": committed_traffic(key, gdom),
                "kernel": gdom.kernel.function_name, "peak_src": src, "algorithmic_flops": kflops}

    e2e = None
    if not (args.no_e2e or args.profile):
        trace("timed steps done")
        e2e = run_e2e(ops, groups, key, shape, world, args, dist, barrier)
        trace("e2e done")

    cpu = None
    if rank == 0 and world == 1 and not (args.no_cpu or args.profile):
        frac = {"c2": 32, "c3": 32, "c3sum": 32, "c4": 32, "c5": 256, "c1": 1}[key]
        t, sshape, used = time_cpu(key, 1, frac)
        cval = amount(key, sshape) / t
        cpu = {"value": cval, "unit": unit, "cores": used, "kind": "port",
               "sample": f"{sshape}: 1/{frac} of the configuration, numpy fp32 restatement (oracle/), 1 thread"}

    if rank == 0:
        line = {
            "metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": hib, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded numpy draws of the config's distributions)",
            "config": {"workload": key, **shape, "parallelism": f"rows/batch sharded x{world}",
                       "kernels": [g.strategy.value for g in groups],
                       "l2": "flushed between steps" if needs_flush else "inputs larger than L2"},
            "e2e": e2e, "roofline": roof, "cpu_baseline": cpu, "clocks": clocks,
            "gpu_launches": args.steps * len(groups), "wall_s": wall, "graph_replay": graph is not None,
            "group_ms": {g.kernel.function_name: m for g, m in zip(groups, group_ms)},
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        distributed.shutdown()
        trace("communicator destroyed")
        dist.destroy_process_group()


def kernel_bytes(g, ops) -> float:
    """Algorithmic bytes of one launch of group ``g``: each bound input buffer read
    once, each output written once (sizes from the IR)."""
    tensors = ops.tensors
    sizes = {}
    for op in ops.build():
        sizes[op.out.buffer_key] = op.out.nbytes
    for n, a in ops.uploads.items():
        sizes[tensors[n].buffer_key] = a.nbytes
    return float(sum(sizes.get(k, 0) for k in dict.fromkeys(g.bindings)))


def kernel_flops(g) -> float:
    from metellus_b200.orchestrator.ir import MatmulOp

    f = 0.0
    for op in g.ops:
        if isinstance(op, MatmulOp):
            M, K = op.a.matrix_shape
            N = op.b.matrix_shape[1]
            f += 2.0 * M * N * K * op.out.batch
    return f


def tensor_peak(g, pk) -> tuple[float, str]:
    if g.pipe == "tcgen05":
        tf32 = pk.get("tf32_tflops")
        if tf32:
            return tf32 / 3.0, "measured tf32_tflops / 3 (3xTF32)"
        return pk.get("bf16_tflops", 1590.0) / 2.0 / 3.0, f"{pk['src']} bf16_tflops / 2 / 3 (tf32 = bf16/2, 3xTF32)"
    return 148 * 128 * 2 * 1.965e9 / 1e12, "FP32 FFMA nominal (148 SMs x 128 lanes x 2 x 1.965 GHz)"


def committed_traffic(key: str, g) -> float | None:
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    d = json.loads(p.read_text())
    return d.get(key, {}).get(g.strategy.value)


def run_e2e(ops, groups, key, shape, world, args, dist, barrier) -> dict:
    """Same program through the public API with host buffers: ``Executable`` (compiled
    once, persistent device buffers, kernels replayed from a CUDA graph) called on
    pinned host inputs, writing the output into a pinned host array; each step's
    host-to-device input copies, kernels and device-to-host output copy are inside the
    CUDA events (a step's download runs on the copy stream, overlapping the next step's
    uploads; the closing event waits for the last one)."""
    from metellus_b200 import distributed
    from metellus_b200.api.executable import Executable
    from metellus_b200.runtime import backend

    out_name = configs.CONFIGS[key].output
    combine = (out_name,) if key == "c3sum" and world > 1 else ()
    with distributed.combining(*combine):
        exe = Executable(ops, outputs=(out_name,))
    pinned = {}
    for n, a in ops.uploads.items():
        pa = backend.PinnedArray(a.shape)
        pa.array[...] = a
        pinned[n] = pa
    out_host = backend.PinnedArray(ops.tensors[out_name].shape)
    inputs = {n: p.array for n, p in pinned.items()}
    outs = {out_name: out_host.array}

    # programs with an NCCL combine wait for the device at the end of every step (an
    # 8-rank run that queued such steps back to back without waiting stalled)
    wait_each = any("nccl" in (g.pipe or "") for g in exe.groups)

    def step():
        exe(inputs, out=outs, wait=wait_each)

    steps = max(3, min(args.steps, 10))
    trace = os.environ.get("METELLUS_TRACE")
    for i in range(3):
        step()
        if trace:
            exe.synchronize()
            print(f"[rank {os.environ.get('RANK', '0')}] e2e warm-up step {i} done", file=sys.stderr, flush=True)
    exe.synchronize()
    barrier()
    e0, e1 = backend.Event(), backend.Event()
    e0.record()
    for _ in range(steps):
        step()
    exe.join()  # the last step's download (copy stream) inside the timed region
    e1.record()
    barrier()
    exe.synchronize()
    ms = e0.elapsed_ms(e1) / steps
    if dist is not None:
        import torch

        t = torch.tensor([ms], device=f"cuda:{int(os.environ.get('LOCAL_RANK', '0'))}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    h2d = int(sum(p.array.nbytes for p in pinned.values()))
    d2h = int(out_host.array.nbytes)
    exe.close()
    _, unit, _ = metric_of(key)
    return {"value": amount(key, shape) * world / (ms / 1e3), "unit": unit, "ms_per_step": ms,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "api": "metellus_b200.Executable"}


if __name__ == "__main__":
    main()
