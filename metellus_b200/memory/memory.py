"""Cooperative global <-> shared tile copies (reference: src/memory/memory.py:359-517).

Semantics kept from the reference: a load applies ``value_transform`` to in-bounds
reads only and writes 0.0f for out-of-bounds elements (the matmul / sum identity,
memory.py:8-11, 157); 128-bit vector copies are used when the tile's column count is
a multiple of 4 and the global column stride is the literal "1".

CUDA specifics: addresses are computed in 64-bit (``size_t``) so tensors above 2^32
elements index correctly; a load may write the tile *transposed*
(``dst[tile_col][tile_row]``), which the SIMT matmul uses so both operand tiles are
read with conflict-free 128-bit shared loads in the inner product loop.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

from metellus_b200.compute.fragments import CodegenContext, TgmemAccess

ValueTransform = Callable[[str], str]


def _col_term(stride: str) -> str:
    return "global_col" if stride == "1" else f"(size_t)global_col * ({stride})"


def tg_load(
    src_name: str,
    src_row_stride: str,
    row_start: str,
    col_start: str,
    dst_name: str,
    tile_shape: tuple[int, int],
    num_threads: int,
    row_limit: str | None = None,
    col_limit: str | None = None,
    src_col_stride: str = "1",
    value_transform: ValueTransform | None = None,
    transpose: bool = False,
) -> str:
    rows, cols = tile_shape
    tf = value_transform or (lambda e: e)
    checked = row_limit is not None and col_limit is not None
    dst = (lambda r, c: f"{dst_name}[{c}][{r}]") if transpose else (lambda r, c: f"{dst_name}[{r}][{c}]")
    row_addr = f"(size_t)global_row * ({src_row_stride})"
    vec = cols % 4 == 0 and src_col_stride == "1"
    if not vec:
        raw = f"{src_name}[{row_addr} + {_col_term(src_col_stride)}]"
        val = tf(raw)
        if checked:
            val = f"(global_row < ({row_limit}) && global_col < ({col_limit})) ? ({val}) : 0.0f"
        return (
            f"for (unsigned idx = flat_tid; idx < {rows * cols}u; idx += {num_threads}u) {{\n"
            f"    const unsigned tile_row = idx / {cols}u, tile_col = idx % {cols}u;\n"
            f"    const unsigned global_row = ({row_start}) + tile_row;\n"
            f"    unsigned global_col = ({col_start}) + tile_col;\n"
            f"    {dst('tile_row', 'tile_col')} = {val};\n"
            f"}}"
        )
    c4 = cols // 4
    addr = f"{src_name} + {row_addr} + global_col"
    comps = ("x", "y", "z", "w")
    xf = "".join(
        ("global_col += 1; " if k else "") + f"v.{c} = {tf('v.' + c)}; " for k, c in enumerate(comps)
    ) if value_transform else ""
    if checked:
        lanes = "".join(
            f"if (global_col < ({col_limit})) v.{c} = {tf(src_name + '[' + row_addr + ' + global_col]')}; global_col += 1; "
            for c in comps
        )
        body = (
            f"float4 v = make_float4(0.f, 0.f, 0.f, 0.f);\n"
            f"    if (global_row < ({row_limit})) {{\n"
            f"        if (global_col + 3 < ({col_limit}) && (({row_addr} + global_col) & 3) == 0) {{\n"
            f"            v = *reinterpret_cast<const float4*>({addr}); {xf}\n"
            f"        }} else {{ {lanes} }}\n"
            f"    }}"
        )
    else:
        body = f"float4 v = *reinterpret_cast<const float4*>({addr}); {xf}"
    stores = " ".join(f"{dst('tile_row', f'tile_col + {k}')} = v.{c};" for k, c in enumerate(comps))
    return (
        f"for (unsigned idx = flat_tid; idx < {rows * c4}u; idx += {num_threads}u) {{\n"
        f"    const unsigned tile_row = idx / {c4}u, tile_col = (idx % {c4}u) * 4u;\n"
        f"    const unsigned global_row = ({row_start}) + tile_row;\n"
        f"    unsigned global_col = ({col_start}) + tile_col;\n"
        f"    {body}\n"
        f"    {stores}\n"
        f"}}"
    )


def tg_store(
    src_name: str,
    dst_name: str,
    dst_row_stride: str,
    row_start: str,
    col_start: str,
    tile_shape: tuple[int, int],
    num_threads: int,
    row_limit: str | None = None,
    col_limit: str | None = None,
    dst_col_stride: str = "1",
) -> str:
    rows, cols = tile_shape
    checked = row_limit is not None and col_limit is not None
    row_addr = f"(size_t)global_row * ({dst_row_stride})"
    vec = cols % 4 == 0 and dst_col_stride == "1"
    if not vec:
        st = f"{dst_name}[{row_addr} + {_col_term(dst_col_stride)}] = {src_name}[tile_row][tile_col];"
        if checked:
            st = f"if (global_row < ({row_limit}) && global_col < ({col_limit})) {{ {st} }}"
        return (
            f"for (unsigned idx = flat_tid; idx < {rows * cols}u; idx += {num_threads}u) {{\n"
            f"    const unsigned tile_row = idx / {cols}u, tile_col = idx % {cols}u;\n"
            f"    const unsigned global_row = ({row_start}) + tile_row;\n"
            f"    const unsigned global_col = ({col_start}) + tile_col;\n"
            f"    {st}\n"
            f"}}"
        )
    c4 = cols // 4
    vec_expr = (f"make_float4({src_name}[tile_row][tile_col], {src_name}[tile_row][tile_col + 1], "
                f"{src_name}[tile_row][tile_col + 2], {src_name}[tile_row][tile_col + 3])")
    addr = f"{dst_name} + {row_addr} + global_col"
    if checked:
        lanes = " ".join(
            f"if (global_col + {k} < ({col_limit})) {dst_name}[{row_addr} + global_col + {k}] = {src_name}[tile_row][tile_col + {k}];"
            for k in range(4)
        )
        st = (
            f"if (global_row < ({row_limit})) {{\n"
            f"        if (global_col + 3 < ({col_limit}) && (({row_addr} + global_col) & 3) == 0) {{\n"
            f"            *reinterpret_cast<float4*>({addr}) = v;\n"
            f"        }} else {{ {lanes} }}\n"
            f"    }}"
        )
    else:
        st = f"*reinterpret_cast<float4*>({addr}) = v;"
    return (
        f"for (unsigned idx = flat_tid; idx < {rows * c4}u; idx += {num_threads}u) {{\n"
        f"    const unsigned tile_row = idx / {c4}u, tile_col = (idx % {c4}u) * 4u;\n"
        f"    const unsigned global_row = ({row_start}) + tile_row;\n"
        f"    const unsigned global_col = ({col_start}) + tile_col;\n"
        f"    const float4 v = {vec_expr};\n"
        f"    {st}\n"
        f"}}"
    )


@dataclass(frozen=True)
class TgLoadFragment:
    """Global -> shared tile load (memory.py:434-475)."""

    name: str
    src_name: str
    src_row_stride: str
    row_start: str
    col_start: str
    dst_name: str
    tile_shape: tuple[int, int]
    num_threads: int
    row_limit: str | None = None
    col_limit: str | None = None
    src_col_stride: str = "1"
    value_transform: ValueTransform | None = None
    transpose: bool = False
    kind: str = "memory"

    def render(self, ctx: CodegenContext) -> str:
        return tg_load(
            self.src_name, self.src_row_stride, self.row_start, self.col_start, self.dst_name,
            self.tile_shape, self.num_threads, self.row_limit, self.col_limit,
            self.src_col_stride, self.value_transform, self.transpose,
        )

    @property
    def stored_shape(self) -> tuple[int, int]:
        r, c = self.tile_shape
        return (c, r) if self.transpose else (r, c)

    @property
    def tgmem_accesses(self) -> tuple[TgmemAccess, ...]:
        r, c = self.tile_shape
        return (TgmemAccess(self.dst_name, "write", r * c, self.stored_shape),)


@dataclass(frozen=True)
class TgStoreFragment:
    """Shared -> global tile store (memory.py:478-517)."""

    name: str
    src_name: str
    dst_name: str
    dst_row_stride: str
    row_start: str
    col_start: str
    tile_shape: tuple[int, int]
    num_threads: int
    row_limit: str | None = None
    col_limit: str | None = None
    dst_col_stride: str = "1"
    kind: str = "store"

    def render(self, ctx: CodegenContext) -> str:
        return tg_store(
            self.src_name, self.dst_name, self.dst_row_stride, self.row_start, self.col_start,
            self.tile_shape, self.num_threads, self.row_limit, self.col_limit, self.dst_col_stride,
        )

    @property
    def tgmem_accesses(self) -> tuple[TgmemAccess, ...]:
        r, c = self.tile_shape
        return (TgmemAccess(self.src_name, "read", r * c, self.tile_shape),)
