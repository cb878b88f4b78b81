"""Elementwise chain applied in place on a shared-memory tile (reference:
src/compute/elementwise/tiled_chain.py:44-220).

Used by the SIMT matmul shared-tile epilogue and the multi-anchor merge. Secondary
operands come either from another shared tile (``y_tile_for`` / ``cond_tile_for``,
e.g. the second anchor's ``C1_tile``) or straight from global memory at the
element's global (row, col) — on B200 a broadcast bias row is an L1/L2 hit, so it is
not staged through shared memory as the reference does (chain_tiles.py).
"""

from __future__ import annotations

from dataclasses import dataclass, field

from metellus_b200.compute.elementwise import BroadcastSpec, elementwise_expression
from metellus_b200.compute.fragments import CodegenContext, TgmemAccess
from metellus_b200.orchestrator.ir import ElementwiseOp, Scalar, Tensor


def tile_operand_ref(tile: str, broadcast: BroadcastSpec) -> str:
    if broadcast is BroadcastSpec.SCALAR:
        return f"{tile}[0][0]"
    if broadcast is BroadcastSpec.ROW:
        return f"{tile}[0][tile_col]"
    if broadcast is BroadcastSpec.COL:
        return f"{tile}[tile_row][0]"
    return f"{tile}[tile_row][tile_col]"


@dataclass(frozen=True)
class TiledElementwiseChainFragment:
    chain: tuple[ElementwiseOp, ...]
    primary_tile: str
    tile_shape: tuple[int, int]
    num_threads: int
    y_tile_for: dict[int, str]
    cond_tile_for: dict[int, str] = field(default_factory=dict)
    row_origin: str = "0u"
    col_origin: str = "0u"
    row_limit: str | None = None
    col_limit: str | None = None
    name: str = "tiled_elementwise_chain"
    kind: str = "compute"

    def render(self, ctx: CodegenContext) -> str:
        from metellus_b200.orchestrator.assembly.expressions import (
            operand_expr,
            substitute,
            wrap_bool,
        )

        rows, cols = self.tile_shape
        prim = self.chain[0].operands[0]
        cur = f"{self.primary_tile}[tile_row][tile_col]"
        values: dict[str, str] = {}
        if isinstance(prim, Tensor):
            values[prim.name] = cur
        lines = []
        for i, elem in enumerate(self.chain):
            subs = {"x": f"({cur})"}
            for k, key, tiles, mode in ((1, "y", self.y_tile_for, elem.y_broadcast),
                                        (2, "cond", self.cond_tile_for, elem.cond_broadcast)):
                if k >= len(elem.operands):
                    continue
                o = elem.operands[k]
                if isinstance(o, Scalar):
                    subs[key] = f"({operand_expr(o, broadcast=mode, row_var='', col_var='')})"
                elif o.name in values:
                    subs[key] = f"({values[o.name]})"
                elif i in tiles:
                    subs[key] = f"({tile_operand_ref(tiles[i], mode)})"
                else:
                    subs[key] = f"({operand_expr(o, broadcast=mode, row_var='global_row', col_var='global_col')})"
            lines.append(f"const float v{i} = {wrap_bool(elem.op, substitute(elementwise_expression(elem.op), **subs))};")
            cur = f"v{i}"
            values[elem.out.name] = cur
        lines.append(f"{self.primary_tile}[tile_row][tile_col] = {cur};")
        guard = ""
        if self.row_limit is not None:
            guard = f"if (global_row >= ({self.row_limit}) || global_col >= ({self.col_limit})) continue;\n    "
        body = "\n    ".join(lines)
        return (
            f"for (unsigned idx = flat_tid; idx < {rows * cols}u; idx += {self.num_threads}u) {{\n"
            f"    const unsigned tile_row = idx / {cols}u, tile_col = idx % {cols}u;\n"
            f"    const unsigned global_row = ({self.row_origin}) + tile_row, global_col = ({self.col_origin}) + tile_col;\n"
            f"    {guard}{body}\n"
            f"}}"
        )

    @property
    def tgmem_accesses(self) -> tuple[TgmemAccess, ...]:
        r, c = self.tile_shape
        acc = [TgmemAccess(self.primary_tile, "readwrite", r * c, self.tile_shape)]
        for i, elem in enumerate(self.chain):
            for tiles in (self.y_tile_for, self.cond_tile_for):
                if i in tiles:
                    acc.append(TgmemAccess(tiles[i], "read", r * c, self.tile_shape))
        return tuple(acc)
