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


COLRED_WARPS = 8            # warps per block; each walks every 8th reduced index
COLRED_COLS = 128           # outputs per block: 32 lanes x 4 consecutive outputs
COLRED_UNROLL = 4           # reduced indices loaded per thread before folding them


@dataclass(frozen=True)
class ColumnReductionFragment:
    """Last-axis reduction of a view whose *rows* are contiguous (``row_stride`` 1) and
    whose reduced axis strides by ``col_stride`` -- ``reduction(transpose(X))``, the
    reference's way to reduce a row-major X over its first axis (its sandbox test
    "Reduce sum over last axis of a transposed view", sandbox.py:177-186).

    The one-block-per-row template reads such a view one strided element per thread
    (a 32-sector request per warp). Here a block owns 128 consecutive outputs: lane l
    of every warp loads outputs [4l, 4l+4) of one reduced index (a 512-byte coalesced
    row segment, float4 when ``vec``), the 8 warps take every 8th reduced index of the
    block's split, and the warps' partials are combined in shared memory in warp
    order. ``gridDim.y`` splits the reduced axis when the outputs alone do not fill
    the GPU: each split writes its 128 partials to ``partials[split * M + out]`` and
    the last split block of a column block (ticket counter, reset by that block)
    combines them in split order, so the result is deterministic. Same value
    transforms as the row template: ``value_transform`` on each load (variables
    ``row`` = output index, ``idx`` = reduced index), ``epilogue`` on each result."""

    op: str
    input_name: str
    output_name: str
    part_name: str            # splits * M floats (global scratch), unused when splits == 1
    ticket_name: str          # one counter per column block (global scratch, zeroed)
    col_stride: int
    splits: int
    vec: bool
    name: str
    value_transform: ValueTransform | None = None
    epilogue: ValueTransform | None = None
    kind: str = "compute"

    @property
    def tgmem_accesses(self) -> tuple[TgmemAccess, ...]:
        n = COLRED_WARPS * COLRED_COLS
        return (TgmemAccess("colred_sh", "readwrite", n, (COLRED_WARPS, COLRED_COLS)),)

    def _accumulate(self, R: str, q: str, idx: str) -> list[str]:
        """Fold the four values of reduced index ``idx`` (already loaded into ``q``
        when ``vec``) into acc0..acc3."""
        cs = self.col_stride
        lines: list[str] = []
        for l in range(4):
            if self.vec:
                raw = f"{q}.{'xyzw'[l]}"
                val = self.value_transform(raw) if self.value_transform else raw
                lines.append(f"        {{ const unsigned row = row0 + {l}u; const unsigned idx = {idx}; "
                             f"(void)row; (void)idx; acc{l} = {R}::op(acc{l}, {val}); }}")
            else:
                raw = f"{self.input_name}[(size_t)idx * {cs}ull + row]"
                val = self.value_transform(raw) if self.value_transform else raw
                lines.append(f"        {{ const unsigned row = row0 + {l}u; const unsigned idx = {idx}; "
                             f"if (row < M) acc{l} = {R}::op(acc{l}, {val}); }}")
        return lines

    def render(self, ctx: CodegenContext) -> str:
        R = reduction_combiner(self.op)
        W, C = COLRED_WARPS, COLRED_COLS
        fin = "v" if self.epilogue is None else self.epilogue("v")
        out = [
            f"const unsigned lane = flat_tid & 31u, warp_id = flat_tid >> 5;",
            f"const unsigned row0 = tg.x * {C}u + lane * 4u;",
            f"const unsigned split = tg.y;",
            f"const unsigned chunk = (K + {self.splits - 1}u) / {self.splits}u;",
            f"const unsigned i0 = split * chunk;",
            f"const unsigned i1 = (i0 + chunk < K) ? i0 + chunk : K;",
            f"float acc0 = {R}::id(), acc1 = {R}::id(), acc2 = {R}::id(), acc3 = {R}::id();",
        ]
        U = COLRED_UNROLL
        ld = (lambda i: f"__ldcs(reinterpret_cast<const float4*>({self.input_name} + "
                        f"(size_t)({i}) * {self.col_stride}ull + row0))")
        out.append("if (row0 < M) {")
        out.append(f"    unsigned i = i0 + warp_id;")
        if self.vec:
            # U independent 16-byte loads in flight per thread, then the folds
            out.append(f"    for (; i + {(U - 1) * W}u < i1; i += {U * W}u) {{")
            for u in range(U):
                out.append(f"        const float4 q{u} = {ld(f'i + {u * W}u')};")
            for u in range(U):
                out += self._accumulate(R, f"q{u}", f"i + {u * W}u")
            out.append("    }")
            out.append(f"    for (; i < i1; i += {W}u) {{")
            out.append(f"        const float4 q0 = {ld('i')};")
            out += self._accumulate(R, "q0", "i")
            out.append("    }")
        else:
            out.append(f"    #pragma unroll 4")
            out.append(f"    for (; i < i1; i += {W}u) {{")
            out += self._accumulate(R, "", "i")
            out.append("    }")
        out.append("}")
        out += [
            f"*reinterpret_cast<float4*>(&colred_sh[warp_id][lane * 4u]) = make_float4(acc0, acc1, acc2, acc3);",
            f"__syncthreads();",
            f"const unsigned col = tg.x * {C}u + flat_tid;",
            f"float part = {R}::id();",
            f"if (flat_tid < {C}u) {{",
            f"    #pragma unroll",
            f"    for (int w = 0; w < {W}; ++w) part = {R}::op(part, colred_sh[w][flat_tid]);",
            f"}}",
        ]
        if self.splits == 1:
            out += [
                f"if (flat_tid < {C}u && col < M) {{",
                f"    float v = part;",
                f"    v = {fin};",
                f"    {self.output_name}[col] = v;",
                f"}}",
            ]
            return "\n".join(out)
        P, T = self.part_name, self.ticket_name
        out += [
            f"__shared__ bool colred_last;",
            f"if (flat_tid < {C}u && col < M) {P}[(size_t)split * M + col] = part;",
            f"__threadfence();",
            f"__syncthreads();",
            f"if (flat_tid == 0) colred_last = "
            f"(atomicAdd(reinterpret_cast<unsigned*>({T}) + tg.x, 1u) == {self.splits - 1}u);",
            f"__syncthreads();",
            f"if (!colred_last) return;",
            f"__threadfence();",
            f"if (flat_tid < {C}u && col < M) {{",
            f"    float v = {R}::id();",
            f"    for (unsigned s = 0; s < {self.splits}u; ++s) v = {R}::op(v, __ldcg({P} + (size_t)s * M + col));",
            f"    v = {fin};",
            f"    {self.output_name}[col] = v;",
            f"}}",
            f"if (flat_tid == 0) reinterpret_cast<unsigned*>({T})[tg.x] = 0u;  // ready for the next launch",
        ]
        return "\n".join(out)
