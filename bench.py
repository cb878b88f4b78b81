"""Benchmark of the Metellus B200 backend on the BASELINE configurations.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2] [--impl ours|reference]

One step = one run of the whole fused program over one batch of synthetic inputs
(seeded, the configuration's shapes and distributions). Default workload: config C2
(the elementwise DAG, x/y/z fp32 8192x8192), the configuration the metric is quoted
on that fits one GPU; ``--config c1|c3|c3sum|c4|c5`` runs the others.

Multi-GPU (torchrun, one process per GPU): strong scaling. The one full
configuration is split across the ranks by rows (C2, C3, C3-sum, C5) or heads (C4),
weights replicated; the only collective is C3-sum's all-reduce of the partial sums.
C1 has no row or batch dimension to split, so its ranks run replicas. Timing is the
max over ranks of CUDA-event device time, ``value`` = the full configuration's work /
that time. ``weak`` adds the same measurement with the full configuration on every
rank.

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
    p.add_argument("--no-weak", action="store_true", help="N > 1: skip the extra weak-scaling measurement")
    p.add_argument("--shape", default="", help="override the configuration's shape, e.g. M=2048,N=8192 "
                   "(profiling captures on a smaller case)")
    return p.parse_args()


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


def _direct_program(key: str, u: dict):
    """A hand-fused numpy implementation of config ``key`` (not the IR interpreter):
    in-place ufuncs over blocks of rows for the elementwise / row programs, BLAS for the
    products. Returns a callable that runs it once over the arrays ``u``."""
    f32 = np.float32
    if key == "c2":
        x, y, z = u["x"], u["y"], u["z"]

        def block(a, b):
            t = np.multiply(x[a:b], y[a:b])
            t += z[a:b]
            np.tanh(t, out=t)
            t *= f32(0.5)
            e = np.negative(x[a:b])
            np.exp(e, out=e)
            e += f32(1)
            np.reciprocal(e, out=e)
            t += e
            m = np.multiply(z[a:b], f32(0.25))
            np.maximum(m, x[a:b], out=m)
            t -= m
            return t
        return block, x.shape[0]
    if key == "c3":
        X = u["X"]

        def block(a, b):
            e = X[a:b] - X[a:b].max(axis=1, keepdims=True)
            np.exp(e, out=e)
            e /= e.sum(axis=1, keepdims=True)
            return e
        return block, X.shape[0]
    if key == "c3sum":
        X = u["X"]
        return (lambda a, b: X[a:b].sum(dtype=np.float64)), X.shape[0]
    return None, 0


def _direct_blas(key: str, u: dict) -> None:
    """The matmul programs in plain numpy / BLAS (BLAS threads itself)."""
    f32 = np.float32
    if key == "c1":
        np.maximum(u["A"] @ u["B"] + u["bias"], f32(0))
    elif key == "c4":
        for h in range(u["Q"].shape[0]):
            s_ = (u["Q"][h] @ u["K"][h].T) * f32(0.125)
            s_ -= s_.max(axis=1, keepdims=True)
            np.exp(s_, out=s_)
            s_ /= s_.sum(axis=1, keepdims=True)
            _ = s_ @ u["V"][h]
    elif key == "c5":
        X = u["X"]
        c = X - X.mean(axis=1, keepdims=True)
        H = c / np.sqrt((c * c).mean(axis=1, keepdims=True) + f32(1e-5))
        z1 = H @ u["W1"] + u["b1"]
        g = f32(0.5) * z1 * (f32(1) + np.tanh(f32(math.sqrt(2 / math.pi)) * (z1 + f32(0.044715) * z1 ** 3)))
        _ = (g * (H @ u["W3"])) @ u["W2"] + u["b2"] + X


def time_cpu_direct(key: str, frac_rows: int) -> dict:
    """Best-effort CPU time of the same sample as the port baseline: a hand-fused numpy
    program over all host threads (row blocks in a thread pool; BLAS threading for the
    products), best of two runs."""
    threads = os.cpu_count() or 1
    shape = cpu_sample_shape(key, frac_rows)
    u = configs.CONFIGS[key].build(**shape).uploads
    block, rows = _direct_program(key, u)
    best = math.inf
    if block is not None:
        step = max(1, min(64, -(-rows // threads)))
        spans = [(a, min(rows, a + step)) for a in range(0, rows, step)]
        with ThreadPoolExecutor(max_workers=threads) as ex:
            for _ in range(2):
                t0 = time.perf_counter()
                list(ex.map(lambda ab: block(*ab), spans))
                best = min(best, time.perf_counter() - t0)
        how = f"hand-fused numpy over blocks of {step} rows, {threads} threads"
    else:
        for _ in range(2):
            t0 = time.perf_counter()
            _direct_blas(key, u)
            best = min(best, time.perf_counter() - t0)
        how = "numpy with the host BLAS's own threads"
    _, unit, _ = metric_of(key)
    return {"value": amount(key, shape) / best, "unit": unit, "cores": threads, "kind": "numpy direct",
            "sample": f"{shape}: 1/{frac_rows} of the configuration, {how}"}


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
        "scaling": "weak" if configs.SHARD_AXIS[key] is None else "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded)",
        "config": {"workload": key, **shape, "full": configs.CONFIGS[key].full},
        "cpu_baseline": {"value": value, "unit": unit, "cores": used, "kind": "port",
                         "sample": f"{shape} per step (1/{frac} of the configuration), numpy fp32 "
                                   f"restatement of the reference program, {used} host threads"},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# -- GPU arm --------------------------------------------------------------------------------


class Prepared:
    """One program compiled, bound to device buffers and ready to time: its dispatch
    list, an L2-flush buffer when the inputs fit in L2, and (after ``capture``) a CUDA
    graph of one step."""

    def __init__(self, ops, key: str, combine: tuple[str, ...] = ()) -> None:
        from metellus_b200 import distributed
        from metellus_b200.api.run import compile_program
        from metellus_b200.orchestrator.scheduler import buffer_sizes, dispatch_of
        from metellus_b200.runtime.buffer import Buffer

        self.ops = ops
        with distributed.combining(*combine):
            self.groups = compile_program(ops)
        for g in self.groups:
            _ = g.kernel.handle  # compile before timing
        tensors = ops.tensors
        sizes = buffer_sizes(ops, self.groups)
        self.env = {}
        for name, arr in ops.uploads.items():
            self.env[tensors[name].buffer_key] = Buffer.from_numpy(arr)
        self.dispatches = [dispatch_of(g) for g in self.groups]
        for d in self.dispatches:
            for k in d.bindings:
                if k not in self.env:
                    self.env[k] = Buffer.zeros(sizes[k])
        in_bytes = sum(a.nbytes for a in ops.uploads.values())
        self.needs_flush = in_bytes < 2 * L2_BYTES
        self.flush = Buffer(256 * 1024 * 1024) if self.needs_flush else None
        self.graph = None

    def step(self) -> None:
        for d in self.dispatches:
            d.execute(self.env)

    def capture(self) -> None:
        """Record one step as a CUDA graph (after the warm-up has loaded every module),
        so a timed step is one graph launch and the host stays ahead of the device.
        Programs with an NCCL combine run their dispatches directly."""
        from metellus_b200.runtime import backend

        if any("nccl" in (g.pipe or "") for g in self.groups):
            return
        backend.graph_begin()
        try:
            self.step()
        finally:
            self.graph = backend.graph_end()
        backend.graph_launch(self.graph)
        backend.sync()

    def timed_step(self) -> None:
        from metellus_b200.runtime import backend

        if self.graph is not None:
            backend.graph_launch(self.graph)
        else:
            self.step()

    def _flush(self, i: int) -> None:
        from metellus_b200.runtime import backend

        if self.flush is not None:
            backend.fill_buffer(self.flush.handle, i & 0xFF, wait=False)

    def time_steps(self, steps: int) -> list[float]:
        """Device time (ms) of each of ``steps`` steps. The L2 flush of step i runs
        after step i's closing event, so the host enqueues step i + 1 while the flush
        occupies the GPU and no launch gap lands inside a step."""
        from metellus_b200.runtime import backend

        ev = [(backend.Event(), backend.Event()) for _ in range(steps)]
        self._flush(0xFF)
        for i in range(steps):
            ev[i][0].record()
            self.timed_step()
            ev[i][1].record()
            self._flush(i)
        backend.sync()
        return [a.elapsed_ms(b) for a, b in ev]

    def time_kernels(self, steps: int) -> list[float]:
        """Mean device time (ms) of each kernel over ``steps`` steps (same flush)."""
        from metellus_b200.runtime import backend

        gev = [[(backend.Event(), backend.Event()) for _ in self.groups] for _ in range(steps)]
        self._flush(0xFF)
        for i in range(steps):
            for j, d in enumerate(self.dispatches):
                gev[i][j][0].record()
                d.execute(self.env)
                gev[i][j][1].record()
            self._flush(i)
        backend.sync()
        return [statistics.mean(gev[i][j][0].elapsed_ms(gev[i][j][1]) for i in range(steps))
                for j in range(len(self.groups))]

    def close(self) -> None:
        from metellus_b200.runtime import backend

        backend.sync()
        if self.graph is not None:
            backend.graph_destroy(self.graph)
            self.graph = None
        for b in self.env.values():
            b.release()
        self.env = {}
        if self.flush is not None:
            self.flush.release()
            self.flush = None


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
    from metellus_b200.runtime import backend

    def trace(msg: str) -> None:
        if os.environ.get("METELLUS_TRACE"):
            print(f"[rank {rank}] {msg}", file=sys.stderr, flush=True)

    def barrier() -> None:
        backend.sync()
        if dist is not None:
            dist.barrier()

    def max_over_ranks(ms: float) -> float:
        if dist is None:
            return ms
        import torch

        t = torch.tensor([ms], device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    key = args.config
    # binds the GPU; for N > 1 and a combined reduction also creates the NCCL communicator
    distributed.init(nccl=key == "c3sum")
    trace("device and communicator ready")
    overrides = {}
    for kv in filter(None, args.shape.split(",")):
        k, v = kv.split("=")
        overrides[k] = int(v)
    full = {**configs.CONFIGS[key].full, **overrides}
    replicas = configs.SHARD_AXIS[key] is None
    # strong scaling: the one full configuration split across the ranks (rows / heads);
    # C1 has nothing to split, so its ranks are replicas
    ops, shape = configs.shard(key, world, rank, **overrides)
    combine = (configs.CONFIGS[key].output,) if key == "c3sum" and world > 1 else ()
    prep = Prepared(ops, key, combine)
    groups = prep.groups
    trace("compiled and allocated")
    for _ in range(max(args.warmup, 3)):
        prep.step()
    barrier()
    trace("warm-up done")
    prep.capture()
    barrier()
    # Clock sampling covers a ~1 s soak of the same steps right before the timed
    # region and the timed region itself (nvidia-smi samples every 100 ms).
    sampler = ClockSampler(local)
    sampler.start()
    # The soak runs the same number of steps on every rank: a step of a combined
    # reduction holds an NCCL all-reduce, and ranks that each looped "for 1 s" ran
    # different numbers of them and hung. One batch of 8 steps is timed per rank and
    # the largest batch count any rank needs for ~1 s is used everywhere.
    if not args.profile:
        t0 = time.perf_counter()
        for _ in range(8):
            prep.timed_step()
        backend.sync()
        batches = max(0, math.ceil(1.0 / max(time.perf_counter() - t0, 1e-6)) - 1)
        batches = int(max_over_ranks(float(batches)))
        for _ in range(batches):
            for _ in range(8):
                prep.timed_step()
            backend.sync()
    barrier()
    t_wall = time.perf_counter()
    step_ms = prep.time_steps(args.steps)
    barrier()
    wall = time.perf_counter() - t_wall
    clocks = sampler.stop()
    # per-kernel device times (same inputs, same flush), for the roofline of the
    # dominant kernel
    group_ms = prep.time_kernels(args.steps)
    barrier()
    ms = max_over_ranks(statistics.mean(step_ms))
    total = amount(key, full) * (world if replicas else 1)
    value = total / (ms / 1e3)
    metric, unit, hib = metric_of(key)

    # dominant kernel roofline (this rank's shard)
    j = int(np.argmax(group_ms))
    gdom = groups[j]
    pk = peaks()
    if configs.CONFIGS[key].bound == "hbm":
        dom_bytes = kernel_bytes(gdom, ops)
        achieved = dom_bytes / (group_ms[j] / 1e3) / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / pk["hbm_gbs"], "traffic": None if overrides else committed_traffic(key, gdom, world),
                "kernel": gdom.kernel.function_name, "peak_src": f"{pk['src']} hbm_gbs",
                "algorithmic_bytes": dom_bytes}
    else:
        kflops = kernel_flops(gdom)
        achieved = kflops / (group_ms[j] / 1e3) / 1e12
        pipe_peak, src = tensor_peak(gdom, pk)
        roof = {"bound": "tensor", "achieved": achieved, "peak": pipe_peak, "unit": "TFLOP/s",
                "frac": achieved / pipe_peak, "traffic": None if overrides else committed_traffic(key, gdom, world),
                "kernel": gdom.kernel.function_name, "peak_src": src, "algorithmic_flops": kflops}

    # the same full configuration on every rank (weak scaling), for comparison
    weak = None
    if world > 1 and not replicas and not (args.no_weak or args.profile):
        prep.close()
        wops = configs.CONFIGS[key].build(**full, seed=rank)
        wprep = Prepared(wops, key, combine)
        for _ in range(max(args.warmup, 3)):
            wprep.step()
        barrier()
        wprep.capture()
        barrier()
        wms = max_over_ranks(statistics.mean(wprep.time_steps(args.steps)))
        barrier()
        wprep.close()
        weak = {"value": amount(key, full) * world / (wms / 1e3), "unit": unit, "ms_per_step": wms,
                "per_rank": full}
        trace("weak-scaling steps done")
    else:
        prep.close()

    e2e = None
    if not (args.no_e2e or args.profile):
        trace("timed steps done")
        e2e = run_e2e(ops, key, total, world, args, dist, barrier, max_over_ranks)
        trace("e2e done")

    cpu = None
    if rank == 0 and world == 1 and not (args.no_cpu or args.profile):
        frac = {"c2": 32, "c3": 32, "c3sum": 32, "c4": 32, "c5": 256, "c1": 1}[key]
        t, sshape, used = time_cpu(key, 1, frac)
        cval = amount(key, sshape) / t
        cpu = {"value": cval, "unit": unit, "cores": used, "kind": "port",
               "sample": f"{sshape}: 1/{frac} of the configuration, numpy fp32 restatement (oracle/), 1 thread",
               "direct": time_cpu_direct(key, frac)}

    if rank == 0:
        line = {
            "metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": hib,
            "scaling": "weak" if replicas else "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded numpy draws of the config's distributions)",
            "config": {"workload": key, **full, "per_rank": shape,
                       "parallelism": (f"replicas x{world}" if replicas else
                                       f"{configs.SHARD_AXIS[key]} split {world} ways, weights replicated"),
                       "kernels": [g.strategy.value for g in groups],
                       "l2": "flushed between steps" if prep.needs_flush else "inputs larger than L2"},
            "e2e": e2e, "roofline": roof, "cpu_baseline": cpu, "clocks": clocks, "weak": weak,
            "gpu_launches": args.steps * len(groups), "wall_s": wall, "graph_replay": prep.graph is not None
            or not any("nccl" in (g.pipe or "") for g in groups),
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


# tcgen05.mma kind::tf32 issue rate measured on this pool's B200s (148 CTAs, one
# issuing thread each, back-to-back 128 x 128 x 8 MMAs: 64 cycles each, 4096
# flop/clock/SM); profiles/tcgen05_tf32_issue_rate.md. A 3xTF32 product issues three
# MMAs per k step, so its ceiling is a third of this.
TF32_MMA_TFLOPS = 1101.0


def tensor_peak(g, pk) -> tuple[float, str]:
    if g.pipe == "tcgen05":
        return TF32_MMA_TFLOPS / 3.0, ("measured tcgen05 kind::tf32 issue rate / 3 (3xTF32), "
                                       "profiles/tcgen05_tf32_issue_rate.md")
    return 148 * 128 * 2 * 1.965e9 / 1e12, "FP32 FFMA nominal (148 SMs x 128 lanes x 2 x 1.965 GHz)"


def committed_traffic(key: str, g, world: int = 1) -> float | None:
    """DRAM bytes of one launch of the dominant kernel, from the committed ncu capture of
    the full single-GPU configuration; a rank of an N-way split moves 1/N of them."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    d = json.loads(p.read_text())
    v = d.get(key, {}).get(g.strategy.value)
    if v is None:
        return None
    return v / world if configs.SHARD_AXIS[key] is not None else v


def run_e2e(ops, key, total, world, args, dist, barrier, max_over_ranks) -> dict:
    """Same program through the public API with host buffers: ``Executable`` (compiled
    once, persistent device buffers, kernels replayed from a CUDA graph) called on
    pinned host inputs, writing the output into a pinned host array; each step's
    host-to-device input copies, kernels and device-to-host output copy are inside the
    CUDA events (a step's download runs on the copy stream, overlapping the next step's
    uploads; the closing event waits for the last one). Each rank uploads and
    downloads its own shard; ``total`` is the full configuration's work."""
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
    ms = max_over_ranks(e0.elapsed_ms(e1) / steps)
    h2d = int(sum(p.array.nbytes for p in pinned.values()))
    d2h = int(out_host.array.nbytes)
    exe.close()
    for p in (*pinned.values(), out_host):
        p.free()
    _, unit, _ = metric_of(key)
    return {"value": total / (ms / 1e3), "unit": unit, "ms_per_step": ms,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "bytes_per_step_counted": "per rank",
            "api": "metellus_b200.Executable"}


if __name__ == "__main__":
    main()
