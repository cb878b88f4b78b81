"""Last-axis reduction fragments (reference: src/compute/reduction/reduction.py).

Same contract: one block per row, a strided per-thread accumulate with the prologue
``value_transform`` applied to each raw load, a two-level tree, and a store of
``epilogue(result)`` to ``out[row]`` by thread 0. CUDA version: warp-shuffle trees
(``__shfl_xor_sync``) with one shared slot per warp, 256 threads per row.

Op set and identities are the reference's (reduction.py:7, 172-181): sum -> 0,
product -> 1, max -> -inf, min -> +inf.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

from metellus_b200.compute.fragments import CodegenContext, TgmemAccess

REDUCTION_OPS = ("sum", "max", "min", "product")

ValueTransform = Callable[[str], str]

_COMBINER = {"sum": "mt_sum", "product": "mt_prod", "max": "mt_max", "min": "mt_min"}


def reduction_combiner(op: str) -> str:
    if op not in _COMBINER:
        raise ValueError(f"unsupported reduction op: {op}")
    return _COMBINER[op]


def _scratch_floats(tg_x: int) -> int:
    return (tg_x + 31) // 32


@dataclass(frozen=True)
class LastAxisReductionSetupFragment:
    rows_dim: str
    name: str
    kind: str = "setup"

    @property
    def tgmem_accesses(self) -> tuple[TgmemAccess, ...]:
        return ()

    def render(self, ctx: CodegenContext) -> str:
        return (f"const unsigned row = tg.x;\n"
                f"const unsigned warp_lane = flat_tid & 31u, warp_id = flat_tid >> 5;\n"
                f"if (row >= {self.rows_dim}) return;")


@dataclass(frozen=True)
class LastAxisReductionComputeFragment:
    op: str
    input_name: str
    scratch_name: str
    reduce_dim: str
    row_stride: str
    name: str
    tg_x: int
    col_stride: str = "1"
    value_transform: ValueTransform | None = None
    kind: str = "compute"

    @property
    def tgmem_accesses(self) -> tuple[TgmemAccess, ...]:
        n = _scratch_floats(self.tg_x)
        return (TgmemAccess(self.scratch_name, "readwrite", n, (1, n)),)

    def render(self, ctx: CodegenContext) -> str:
        R = reduction_combiner(self.op)
        idx = "idx" if self.col_stride == "1" else f"(size_t)idx * ({self.col_stride})"
        raw = f"{self.input_name}[(size_t)row * ({self.row_stride}) + {idx}]"
        val = self.value_transform(raw) if self.value_transform else raw
        nw = _scratch_floats(self.tg_x)
        S = self.scratch_name
        return (
            f"float acc = {R}::id();\n"
            f"for (unsigned idx = flat_tid; idx < {self.reduce_dim}; idx += {self.tg_x}u) {{\n"
            f"    const float value = {val};\n"
            f"    acc = {R}::op(acc, value);\n"
            f"}}\n"
            f"acc = mt_warp_reduce<{R}>(acc);\n"
            f"if (warp_lane == 0) {S}[warp_id] = acc;\n"
            f"__syncthreads();\n"
            f"if (warp_id == 0) {{\n"
            f"    float r = (warp_lane < {nw}u) ? {S}[warp_lane] : {R}::id();\n"
            f"    r = mt_warp_reduce<{R}>(r);\n"
            f"    if (warp_lane == 0) {S}[0] = r;\n"
            f"}}\n"
            f"__syncthreads();"
        )


@dataclass(frozen=True)
class StoreReductionResultFragment:
    output_name: str
    scratch_name: str
    name: str
    tg_x: int
    value_transform: ValueTransform | None = None
    setup: tuple[str, ...] = ()
    kind: str = "store"

    @property
    def tgmem_accesses(self) -> tuple[TgmemAccess, ...]:
        n = _scratch_floats(self.tg_x)
        return (TgmemAccess(self.scratch_name, "read", n, (1, n)),)

    def render(self, ctx: CodegenContext) -> str:
        lines = [f"float v = {self.scratch_name}[0];", *self.setup]
        if self.value_transform is not None:
            lines.append(f"v = {self.value_transform('v')};")
        lines.append(f"{self.output_name}[row] = v;")
        return "if (flat_tid == 0) {\n    " + "\n    ".join(lines) + "\n}"
