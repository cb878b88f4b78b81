"""Strided gather copy for reshapes that cannot be views (reference:
src/compute/copy/copy.py:26-54 via assembly/shape.py:14-68): output element ``i`` (row
major) reads the source's logical (i / cols, i % cols) through its strides."""

from __future__ import annotations

from dataclasses import dataclass

from metellus_b200.compute.fragments import CodegenContext, TgmemAccess


@dataclass(frozen=True)
class StridedCopyFragment:
    input_name: str
    output_name: str
    input_row_stride: int
    input_col_stride: int
    input_cols: int
    name: str = "strided_copy"
    kind: str = "compute"

    @property
    def tgmem_accesses(self) -> tuple[TgmemAccess, ...]:
        return ()

    def render(self, ctx: CodegenContext) -> str:
        return (
            f"for (size_t gi = (size_t)tg.x * {ctx.tg_x}u + flat_tid; gi < N; gi += (size_t)gridDim.x * {ctx.tg_x}u) {{\n"
            f"    const size_t in_row = gi / {self.input_cols}ull, in_col = gi % {self.input_cols}ull;\n"
            f"    {self.output_name}[gi] = {self.input_name}[in_row * {self.input_row_stride}ll + in_col * {self.input_col_stride}ll];\n"
            f"}}"
        )
