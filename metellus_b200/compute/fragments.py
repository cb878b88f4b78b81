"""Codegen core: context, barrier / alias fragments and the CUDA kernel renderer.

Mirrors the reference's fragment contract (src/compute/fragments.py:13-129): a kernel
is a list of frozen fragment dataclasses with ``render(ctx) -> str`` and
``tgmem_accesses`` (here: shared-memory accesses), assembled by a template into a
``CodegenContext`` and rendered by ``CodegenEngine``.

CUDA specifics of the renderer:

* one ``extern "C" __global__`` function; buffers are pointer parameters in binding
  order, followed by ``mt_dims dims`` passed *by value* (no per-launch dims buffer,
  unlike the reference's fresh uint32 buffer per dispatch, program.py:186).
* shared-memory tiles are declared as ``smem float NAME[R][C];`` pseudo-decls. The
  renderer lays them out in ONE dynamic ``extern __shared__`` arena (16-byte aligned
  offsets) and binds each name as a typed pointer into it, so tiles can exceed the
  48 KB static limit up to the sm_100a opt-in maximum, and the aliasing pass can
  re-type one slot for several tenants.
* batched groups (gridDim.z = batch) rebase every buffer pointer by
  ``blockIdx.z * batch_stride`` before any fragment runs, so fragments index one
  matrix and never see the batch dimension.
"""

from __future__ import annotations

import re
import textwrap
from dataclasses import dataclass
from typing import Any, Literal

KernelFragment = Any
TgmemAccessKind = Literal["read", "write", "readwrite"]


@dataclass(frozen=True)
class TgmemAccess:
    """One named shared-memory object touched by a fragment (fragments.py:13-18)."""

    name: str
    access: TgmemAccessKind
    size_floats: int
    shape: tuple[int, int]


@dataclass(frozen=True)
class CodegenContext:
    """Everything the renderer needs besides the fragment list.

    ``buffers``: parameter decls in slot order (``const float* __restrict__ X``).
    ``batch_strides``: per-buffer element stride applied per ``blockIdx.z`` (empty
    means unbatched). ``threadgroup_decls``: ``smem float NAME[..]..;`` decls.
    ``extra_params``: trailing parameters after ``dims`` (TMA tensor maps).
    ``static_smem_bytes``: bytes the kernel reserves itself at the arena head
    (mbarriers, TMEM slot) before the tile decls."""

    function_name: str
    buffers: tuple[str, ...]
    dims: tuple[str, ...]
    tg_x: int
    tg_y: int
    threadgroup_decls: tuple[str, ...] = ()
    helpers: tuple[str, ...] = ()
    preamble: tuple[str, ...] = ()
    dims_buffer_index: int | None = None
    batch_strides: tuple[int, ...] = ()
    extra_params: tuple[str, ...] = ()
    static_smem_bytes: int = 0
    min_blocks_per_sm: int = 0

    @property
    def num_threads(self) -> int:
        return self.tg_x * self.tg_y


@dataclass(frozen=True)
class BarrierFragment:
    """Block-wide barrier (fragments.py:37-47)."""

    name: str = "barrier"
    kind: str = "barrier"

    def render(self, ctx: CodegenContext) -> str:
        return "__syncthreads();"

    @property
    def is_tgmem_barrier(self) -> bool:
        return True

    @property
    def tgmem_accesses(self) -> tuple[TgmemAccess, ...]:
        return ()


@dataclass(frozen=True)
class AliasFragment:
    """Re-type a shared-memory slot for its next tenant (fragments.py:51-93).

    Emits a block barrier first unless the template already placed one right
    before, because every thread must be done with the previous tenant."""

    old_name: str
    new_name: str
    new_shape: tuple[int, int]
    preceded_by_barrier: bool
    name: str = "alias"
    kind: str = "alias"

    def render(self, ctx: CodegenContext) -> str:
        cols = self.new_shape[1]
        line = f"float (*{self.new_name})[{cols}] = reinterpret_cast<float (*)[{cols}]>({self.old_name});"
        return line if self.preceded_by_barrier else "__syncthreads();\n" + line

    @property
    def tgmem_accesses(self) -> tuple[TgmemAccess, ...]:
        return ()


_SMEM_DECL_RE = re.compile(r"^\s*smem\s+float\s+(\w+)\s*((?:\[\s*\d+\s*\])+)\s*;\s*$")


def parse_smem_decl(decl: str) -> tuple[str, tuple[int, ...]]:
    """``smem float NAME[a][b];`` -> (NAME, (a, b)). Raises on any other form."""
    m = _SMEM_DECL_RE.match(decl)
    if m is None:
        raise ValueError(f"cannot parse shared-memory decl {decl!r}; expected `smem float <name>[N]...;`")
    dims = tuple(int(x) for x in re.findall(r"\[\s*(\d+)\s*\]", m.group(2)))
    return m.group(1), dims


def smem_layout(decls: tuple[str, ...], head: int = 0) -> tuple[list[tuple[str, tuple[int, ...], int]], int]:
    """Assign 16-byte aligned arena offsets to shared-memory decls; returns
    ([(name, dims, offset)], total_bytes)."""
    out = []
    off = (head + 15) // 16 * 16
    for d in decls:
        name, dims = parse_smem_decl(d)
        n = 1
        for x in dims:
            n *= x
        out.append((name, dims, off))
        off += (4 * n + 15) // 16 * 16
    return out, off


def smem_bytes_of(ctx: CodegenContext) -> int:
    return smem_layout(ctx.threadgroup_decls, ctx.static_smem_bytes)[1]


class CodegenEngine:
    """Render fragments + context into one CUDA C++ kernel (fragments.py:96-129)."""

    def render(self, fragments: list[KernelFragment], ctx: CodegenContext) -> str:
        from metellus_b200.compute.device_lib import DEVICE_PRELUDE

        params = [*ctx.buffers, "const mt_dims dims", *ctx.extra_params]
        lines: list[str] = []
        lines += [f"const unsigned {n} = dims.d[{i}];" for i, n in enumerate(ctx.dims)]
        lines += [
            "const uint3 tg = blockIdx;",
            "const uint3 lid = threadIdx;",
            f"const unsigned flat_tid = threadIdx.y * {ctx.tg_x}u + threadIdx.x;",
        ]
        if ctx.batch_strides:
            for decl, bs in zip(ctx.buffers, ctx.batch_strides):
                if bs:
                    pname = decl.split()[-1]
                    lines.append(f"{pname} += (size_t)blockIdx.z * {bs}ull;")
        layout, total = smem_layout(ctx.threadgroup_decls, ctx.static_smem_bytes)
        if total > 0:
            lines.append("extern __shared__ __align__(1024) unsigned char mt_smem[];")
        for name, dims, off in layout:
            if len(dims) == 1:
                lines.append(f"float* {name} = reinterpret_cast<float*>(mt_smem + {off});")
            else:
                tail = "".join(f"[{d}]" for d in dims[1:])
                lines.append(f"float (*{name}){tail} = reinterpret_cast<float (*){tail}>(mt_smem + {off});")
        lines += list(ctx.preamble)
        for frag in fragments:
            text = frag.render(ctx)
            if text.strip():
                lines.append(text)
        body = textwrap.indent("\n".join(lines), "    ")
        helpers = "\n".join(h.strip() for h in ctx.helpers if h.strip())
        nt = ctx.num_threads
        bounds = f"__launch_bounds__({nt}, {ctx.min_blocks_per_sm})" if ctx.min_blocks_per_sm else f"__launch_bounds__({nt})"
        joined = ",\n    ".join(params)
        return (
            f"{DEVICE_PRELUDE}\n{helpers}\n"
            f"extern \"C\" __global__ void {bounds} {ctx.function_name}(\n    {joined}\n) {{\n{body}\n}}\n"
        )
