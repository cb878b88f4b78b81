"""Multi-GPU host logic on CPU: row sharding, the NCCL-id exchange over a
world-size-2 gloo group, and the plan of a combined (sharded whole-tensor)
reduction. The device-side combine runs in tests/test_gpu_distributed.py."""

from __future__ import annotations

import os

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from metellus_b200 import configs, distributed
from metellus_b200.api.run import compile_program
from metellus_b200.orchestrator.assembly.reduction import PARTIAL_KEY


@pytest.mark.parametrize("n,world", [(32768, 8), (10, 3), (5, 8), (1, 1)])
def test_row_range_partitions_rows(n, world):
    spans = [distributed.row_range(n, r, world) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    sizes = [b - a for a, b in spans]
    assert max(sizes) - min(sizes) <= 1


def test_row_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        distributed.row_range(10, 3, 3)


def _exchange(rank: int, world: int, port: int, q) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        info = distributed.rank_info()
        uid = distributed.exchange_nccl_id(info, make_id=lambda: bytes(range(128)))
        q.put((rank, uid))
    finally:
        dist.destroy_process_group()


def test_nccl_id_exchange_gloo_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_exchange, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got[0] == got[1] == bytes(range(128))


def test_combined_reduction_plan():
    c = configs.CONFIGS["c3sum"]
    ops = c.build(**c.small, materialize=False)
    plain = compile_program(ops)
    assert [g.pipe for g in plain] == ["native"]
    with distributed.combining("total"):
        comb = compile_program(ops)
    assert [g.pipe for g in comb] == ["native+nccl"]
    assert comb[0].kernel.entry == "mt_reduce_rows+mt_allreduce_f64"
    assert dict(comb[0].scratch)[PARTIAL_KEY] == 8


def test_combined_reduction_must_be_standalone():
    from metellus_b200 import Operations

    ops = Operations()
    ops.input("X", (4, 1 << 16))
    ops.elementwise("exp", out="E", operands=("X",))
    ops.reduction("sum", out="S", x="E", axis=-1)
    with distributed.combining("S"), pytest.raises(ValueError, match="combined across GPUs"):
        compile_program(ops)


def test_combined_reduction_rejects_several_rows():
    """Per-row partials of a row-sharded tensor cannot be combined element-wise
    (row i of two shards are different rows), so only whole-tensor reductions combine."""
    from metellus_b200 import Operations

    ops = Operations()
    ops.input("X", (4, 1 << 16))
    ops.reduction("sum", out="S", x="X", axis=-1)
    with distributed.combining("S"), pytest.raises(ValueError, match="single row"):
        compile_program(ops)


def _agree_rank(rank: int, world: int, port: int, q) -> None:
    """Rank 1 holds a shard that cannot be combined (4 rows); rank 0's is fine. Both
    must raise while planning, before any collective would be launched."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from metellus_b200 import Operations

    try:
        ops = Operations()
        ops.input("X", (1, 1 << 16) if rank == 0 else (4, 1 << 14))
        ops.reduction("sum", out="S", x="X", axis=-1)
        try:
            with distributed.combining("S"):
                compile_program(ops)
            q.put((rank, "planned"))
        except ValueError as e:
            q.put((rank, str(e)))
    finally:
        dist.destroy_process_group()


def test_combined_reduction_all_ranks_reject_together():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 30500 + os.getpid() % 1000
    procs = [ctx.Process(target=_agree_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert "rank 1 cannot take part" in got[0], got
    assert "rank 1 cannot take part" in got[1], got
