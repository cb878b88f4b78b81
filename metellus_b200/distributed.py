"""Multi-GPU execution: one process per GPU (launched by torchrun), weak scaling.

Programs with a leading batch / row dimension are sharded by rows across the ranks,
weights replicated: every kernel runs on its rank's shard and nothing is exchanged.
A whole-tensor reduction over a sharded tensor (``sum(X)`` with X's rows split) is the
one program shape that needs a collective: each rank reduces its shard to one fp64
partial (``mt_reduce_rows``, fp64 output) and the partials are combined by a single
NCCL all-reduce over NVLink (``mt_allreduce_f64``), which also writes the fp32
result into the program's output tensor on every rank. Which reduction outputs are
combined is stated by the caller::

    info = distributed.init()                      # binds the GPU, creates the communicator
    with distributed.combining("total"):
        groups = compile_program(ops)              # ops built on this rank's shard

``torch.distributed`` is host plumbing only (rendezvous, broadcasting the NCCL id).
"""

from __future__ import annotations

import contextlib
import contextvars
import os
from dataclasses import dataclass

from metellus_b200.runtime import backend


@dataclass(frozen=True)
class RankInfo:
    rank: int
    world: int
    local_rank: int


def rank_info() -> RankInfo:
    """This process's place in the job, from the torchrun environment."""
    return RankInfo(rank=int(os.environ.get("RANK", "0")), world=int(os.environ.get("WORLD_SIZE", "1")),
                    local_rank=int(os.environ.get("LOCAL_RANK", "0")))


def row_range(n_rows: int, rank: int, world: int) -> tuple[int, int]:
    """[start, stop) of ``rank``'s contiguous block of rows; the first ``n_rows %
    world`` ranks take one row more."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    base, extra = divmod(n_rows, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


_nccl_ready = False


def exchange_nccl_id(info: RankInfo, group=None, make_id=None) -> bytes:
    """Rank 0 creates the NCCL unique id; every rank returns it (broadcast over the
    default torch.distributed group)."""
    import torch.distributed as dist

    make_id = make_id or backend.nccl_unique_id
    obj = [make_id() if info.rank == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    return obj[0]


def init(group=None, *, nccl: bool = True) -> RankInfo:
    """Bind this process to its GPU and, for more than one rank and ``nccl``, create the
    NCCL communicator the combining reductions use (torch.distributed must already be
    initialised then). Programs without a combined reduction pass ``nccl=False``."""
    global _nccl_ready
    info = rank_info()
    backend.set_device(info.local_rank)
    backend.init()
    if nccl and info.world > 1 and not _nccl_ready:
        backend.nccl_init(info.world, info.rank, exchange_nccl_id(info, group))
        _nccl_ready = True
    return info


def shutdown() -> None:
    global _nccl_ready
    if _nccl_ready:
        backend.nccl_destroy()
        _nccl_ready = False


def nccl_ready() -> bool:
    return _nccl_ready


_combined: contextvars.ContextVar[frozenset[str]] = contextvars.ContextVar("metellus_combined", default=frozenset())


@contextlib.contextmanager
def combining(*names: str):
    """Within the block, the reductions producing ``names`` are planned as sharded
    whole-tensor reductions: local fp64 partial + NCCL all-reduce."""
    token = _combined.set(_combined.get() | frozenset(names))
    try:
        yield
    finally:
        _combined.reset(token)


def combined_outputs() -> frozenset[str]:
    return _combined.get()


def agree(problem: str | None, what: str, group=None) -> None:
    """Raise ``ValueError`` on every rank if any rank reports a problem.

    Called while planning a step that ends in a collective: a rank that raised alone
    would leave the others waiting in that collective. The verdicts travel over the
    host process group (``torch.distributed``); without one (a single process) the
    local verdict decides."""
    problems = [problem]
    try:
        import torch.distributed as dist

        if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
            problems = [None] * dist.get_world_size(group)
            dist.all_gather_object(problems, problem, group=group)
    except ImportError:
        pass
    bad = [(r, p) for r, p in enumerate(problems) if p]
    if bad:
        r, p = bad[0]
        raise ValueError(f"{what}: rank {r} cannot take part: {p}" if len(problems) > 1 else p)
