"""Sharded whole-tensor sum on 2, 4 and 8 GPUs (as many as the box has): each rank reduces its shard of X to an fp64
partial and one NCCL all-reduce combines them (``distributed.combining``). Both ranks
must return the fp64 sum of the full tensor rounded once. Runs as child processes,
one per GPU; a world size larger than the box's GPU count is skipped."""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

SHAPE = dict(M=512, K=4096)


def _rank(rank: int, world: int, port: int, q) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    from metellus_b200 import configs, distributed, run

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        distributed.init()
        ops = configs.CONFIGS["c3sum"].build(**SHAPE, seed=rank)
        with distributed.combining("total"):
            res = run(ops)
        q.put((rank, float(res.env["total"].reshape(-1)[0]), [g.pipe for g in res.groups]))
        distributed.shutdown()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_sum(world):
    from metellus_b200 import configs

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 1000
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in procs:
        r, v, pipes = q.get(timeout=300)
        got[r] = (v, pipes)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    ref = sum(configs.CONFIGS["c3sum"].build(**SHAPE, seed=r).uploads["X"].astype(np.float64).sum()
              for r in range(world))
    for r in range(world):
        v, pipes = got[r]
        assert pipes == ["native+nccl"]
        assert abs(v - np.float32(ref)) <= np.spacing(np.float32(abs(ref))), (r, v, ref)
