"""Measured pipe and tile choice for matmul groups.

A matmul group can run on the SIMT FFMA tile (``compute/matmul.py``) or on the
tcgen05 3xTF32 kernel in one of three tilings: ``pair`` (256 x 128 per two-CTA
cluster, ``cta_group::2``), ``one`` (128 x BN on one CTA) or ``splitk`` (128 x 128 on a
two-CTA cluster that splits K). ``pipe_table.json`` next to this file holds, for a
grid of shapes, the device time of every variant measured on a B200 and the fastest
one; ``measure_pipe_table.py`` regenerates it. The reference chooses its single
Metal tile by a fixed rule (src/compute/matmul/config.py:40-51); here the rule
(tensor maps able to describe the operands, then the tile heuristics in
``tc_matmul``) is only the fallback for shapes the table does not cover.

Lookup: an exact (M, N, K, anchors) entry, else the nearest measured shape with the
same number of anchors whose M, N and K are each within a factor of two (nearest in
log2 distance). A pick the operands cannot take (FFMA when a prologue needs the
tensor-core path, a tiling the layout does not allow) falls back to the rule.
"""

from __future__ import annotations

import contextlib
import contextvars
import json
import math
from dataclasses import dataclass
from functools import lru_cache
from pathlib import Path

TABLE_PATH = Path(__file__).with_name("pipe_table.json")
VARIANTS = ("ffma", "one", "splitk", "pair")


@dataclass(frozen=True)
class Pick:
    variant: str          # one of VARIANTS
    source: str           # "table" | "table-near" | "forced"

    @property
    def pipe(self) -> str:
        return "ffma" if self.variant == "ffma" else "tcgen05"


_forced: contextvars.ContextVar[str | None] = contextvars.ContextVar("metellus_forced_variant", default=None)


@contextlib.contextmanager
def forced(variant: str):
    """Plan every matmul in the block with ``variant`` (the measurement uses this)."""
    if variant not in VARIANTS:
        raise ValueError(f"unknown matmul variant {variant!r}; expected one of {VARIANTS}")
    token = _forced.set(variant)
    try:
        yield
    finally:
        _forced.reset(token)


@lru_cache(maxsize=4)
def _load(path: str) -> tuple[dict, ...]:
    p = Path(path)
    if not p.exists():
        return ()
    return tuple(json.loads(p.read_text()).get("entries", ()))


def entries() -> tuple[dict, ...]:
    return _load(str(TABLE_PATH))


def lookup(M: int, N: int, K: int, anchors: int = 1) -> Pick | None:
    """The measured pick for this shape (see the module docstring), or None."""
    v = _forced.get()
    if v is not None:
        return Pick(v, "forced")
    best, best_d = None, math.inf
    for e in entries():
        m, n, k, nb = e["shape"]
        if nb != anchors:
            continue
        d = [abs(math.log2(a / b)) for a, b in ((M, m), (N, n), (K, k))]
        if max(d) > 1.0:
            continue
        dist = sum(d)
        if dist < best_d:
            best, best_d = e, dist
    if best is None:
        return None
    return Pick(best["best"], "table" if best_d == 0 else "table-near")
