"""SIMT (FFMA) matmul tile fragments — the fallback pipe for matmul groups that the
tcgen05 path does not take (prologue transforms on operand loads, shapes that are not
tile-aligned, tiny problems).

Fragment roles follow the reference chain (src/compute/matmul/matmul.py:37-352):
setup -> k-chunk mainloop {load A, load B, barrier, compute, barrier} -> register
epilogue / accumulators to shared tile / shared tile to global. The arithmetic is
CUDA-native: each thread owns a ``tm x tn`` register micro-tile built from 4x4
sub-blocks spread across the CTA tile, the A tile is stored transposed
(``A_tile[k][m]``) so both operands are read with 128-bit shared loads, and products
accumulate with explicit ``fmaf`` (single rounding per step).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable

from metellus_b200.compute.fragments import CodegenContext, TgmemAccess

ValueTransform = Callable[[str], str]
KernelFragment = Any


@dataclass(frozen=True)
class TileConfig:
    tile_M: int
    tile_N: int
    tile_K: int
    tm: int = 4
    tn: int = 4
    a_pad: int = 4
    b_pad: int = 4
    c_pad: int = 1

    @property
    def threads_m(self) -> int:
        return self.tile_M // self.tm

    @property
    def threads_n(self) -> int:
        return self.tile_N // self.tn

    @property
    def num_threads(self) -> int:
        return self.threads_m * self.threads_n

    @property
    def tg_x(self) -> int:
        return self.num_threads

    @property
    def tg_y(self) -> int:
        return 1

    def row_of(self, i: int) -> str:
        """Row within the CTA tile of accumulator row ``i`` of this thread."""
        sub = self.tile_M // (self.tm // 4)
        return f"({(i // 4) * sub + i % 4}u + t_row * 4u)"

    def col_of(self, j: int) -> str:
        sub = self.tile_N // (self.tn // 4)
        return f"({(j // 4) * sub + j % 4}u + t_col * 4u)"


def ceil_div(a: int, b: int) -> int:
    return (a + b - 1) // b


TILE_128 = TileConfig(128, 128, 8, tm=8, tn=8)
TILE_64 = TileConfig(64, 64, 16)
TILE_32 = TileConfig(32, 32, 16)


def select_tile_config(M: int, K: int, N: int, sms: int = 148) -> TileConfig:
    """Largest SIMT tile that still gives about one CTA per SM (the reference picks
    Apple-specific tiles at config.py:40-51)."""
    if ceil_div(M, 128) * ceil_div(N, 128) >= sms:
        return TILE_128
    if M >= 64 and N >= 64:
        return TILE_64
    return TILE_32


def is_aligned_shape(M: int, K: int, N: int, config: TileConfig) -> bool:
    return (M % config.tile_M == 0 and N % config.tile_N == 0 and K % config.tile_K == 0
            and K % 4 == 0 and N % 4 == 0)


def grid_for(M: int, N: int, config: TileConfig) -> tuple[int, int, int]:
    return (ceil_div(N, config.tile_N), ceil_div(M, config.tile_M), 1)


@dataclass(frozen=True)
class MatmulConfig:
    tile: TileConfig
    aligned: bool
    M_dim_var: str
    K_dim_var: str
    N_dim_var: str
    a_buffer_name: str
    b_buffer_name: str
    c_buffer_name: str
    a_tile_name: str
    b_tile_name: str
    c_tile_name: str
    c_col_stride: str = "1"


@dataclass(frozen=True)
class MatmulTileMappingFragment:
    """Block -> tile mapping. ``tg`` (blockIdx) is declared by the renderer."""

    name: str = "tile_mapping"
    kind: str = "setup"

    def render(self, ctx: CodegenContext) -> str:
        return ""

    @property
    def tgmem_accesses(self) -> tuple[TgmemAccess, ...]:
        return ()


@dataclass(frozen=True)
class ThreadIndexFragment:
    tile: TileConfig
    name: str = "thread_index"
    kind: str = "setup"

    def render(self, ctx: CodegenContext) -> str:
        return (f"const unsigned t_row = flat_tid / {self.tile.threads_n}u;\n"
                f"const unsigned t_col = flat_tid % {self.tile.threads_n}u;")

    @property
    def tgmem_accesses(self) -> tuple[TgmemAccess, ...]:
        return ()


@dataclass(frozen=True)
class MatmulSetupFragment:
    config: MatmulConfig
    accumulator_suffix: str = ""
    emit_thread_coords: bool = True
    name: str = "matmul_setup"
    kind: str = "setup"

    def render(self, ctx: CodegenContext) -> str:
        t = self.config.tile
        return f"float acc{self.accumulator_suffix}[{t.tm}][{t.tn}] = {{}};"

    @property
    def tgmem_accesses(self) -> tuple[TgmemAccess, ...]:
        return ()


def _indent(code: str, n: int) -> str:
    return "\n".join((" " * n + ln) if ln else ln for ln in code.splitlines())


@dataclass(frozen=True)
class MatmulMainloopFragment:
    tile_K: int
    fragments: tuple[KernelFragment, ...]
    K_dim_var: str
    name: str = "matmul_mainloop"
    kind: str = "compute"

    def render(self, ctx: CodegenContext) -> str:
        body = "\n".join(f.render(ctx) for f in self.fragments)
        return (f"for (unsigned k_chunk = 0; k_chunk < {self.K_dim_var}; k_chunk += {self.tile_K}u) {{\n"
                f"{_indent(body, 4)}\n}}")

    @property
    def tgmem_accesses(self) -> tuple[TgmemAccess, ...]:
        return ()

    @property
    def sub_fragments(self) -> tuple[KernelFragment, ...]:
        return self.fragments


@dataclass(frozen=True)
class MatmulComputeFragment:
    """Rank-``tile_K`` update of this thread's register micro-tile."""

    config: MatmulConfig
    accumulator_suffix: str = ""
    name: str = "matmul_compute"
    kind: str = "compute"

    def render(self, ctx: CodegenContext) -> str:
        t = self.config.tile
        suf = self.accumulator_suffix
        A, B = self.config.a_tile_name, self.config.b_tile_name
        a_sub = t.tile_M // (t.tm // 4)
        b_sub = t.tile_N // (t.tn // 4)
        loads = []
        for s in range(t.tm // 4):
            loads.append(f"const float4 a{s} = *reinterpret_cast<const float4*>(&{A}[kk][{s * a_sub}u + t_row * 4u]);")
        for s in range(t.tn // 4):
            loads.append(f"const float4 b{s} = *reinterpret_cast<const float4*>(&{B}[kk][{s * b_sub}u + t_col * 4u]);")
        comp = ("x", "y", "z", "w")
        fmas = []
        for i in range(t.tm):
            for j in range(t.tn):
                av = f"a{i // 4}.{comp[i % 4]}"
                bv = f"b{j // 4}.{comp[j % 4]}"
                fmas.append(f"acc{suf}[{i}][{j}] = fmaf({av}, {bv}, acc{suf}[{i}][{j}]);")
        inner = "\n    ".join(loads + fmas)
        return f"#pragma unroll\nfor (unsigned kk = 0; kk < {t.tile_K}u; ++kk) {{\n    {inner}\n}}"

    @property
    def tgmem_accesses(self) -> tuple[TgmemAccess, ...]:
        t = self.config.tile
        return (
            TgmemAccess(self.config.a_tile_name, "read", t.tile_K * (t.tile_M + t.a_pad),
                        (t.tile_K, t.tile_M + t.a_pad)),
            TgmemAccess(self.config.b_tile_name, "read", t.tile_K * (t.tile_N + t.b_pad),
                        (t.tile_K, t.tile_N + t.b_pad)),
        )


@dataclass(frozen=True)
class MatmulRegisterEpilogueFragment:
    """Apply a lane-agnostic transform to every accumulator register (matmul.py:186-234)."""

    config: MatmulConfig
    value_transform: ValueTransform | None = None
    setup: tuple[str, ...] = ()
    accumulator_suffix: str = ""
    name: str = "matmul_register_epilogue"
    kind: str = "compute"

    def render(self, ctx: CodegenContext) -> str:
        if self.value_transform is None and not self.setup:
            return ""
        t = self.config.tile
        lines = list(self.setup)
        if self.value_transform is not None:
            e = f"acc{self.accumulator_suffix}[i][j]"
            lines.append(
                f"#pragma unroll\nfor (int i = 0; i < {t.tm}; ++i) {{\n"
                f"#pragma unroll\n    for (int j = 0; j < {t.tn}; ++j) {{ {e} = {self.value_transform(e)}; }}\n}}"
            )
        return "\n".join(lines)

    @property
    def tgmem_accesses(self) -> tuple[TgmemAccess, ...]:
        return ()


@dataclass(frozen=True)
class MatmulAccumToDevFragment:
    """Aligned fast path: 128-bit stores of the micro-tile straight to global."""

    config: MatmulConfig
    name: str = "matmul_accum_to_dev"
    kind: str = "store"

    def render(self, ctx: CodegenContext) -> str:
        if not self.config.aligned:
            raise ValueError("MatmulAccumToDevFragment requires config.aligned=True")
        t = self.config.tile
        C, N = self.config.c_buffer_name, self.config.N_dim_var
        out = [f"const unsigned c_row0 = tg.y * {t.tile_M}u, c_col0 = tg.x * {t.tile_N}u;"]
        for i in range(t.tm):
            for s in range(t.tn // 4):
                j = 4 * s
                out.append(
                    f"*reinterpret_cast<float4*>({C} + (size_t)(c_row0 + {t.row_of(i)}) * {N} + c_col0 + {t.col_of(j)}) = "
                    f"make_float4(acc[{i}][{j}], acc[{i}][{j + 1}], acc[{i}][{j + 2}], acc[{i}][{j + 3}]);"
                )
        return "\n".join(out)

    @property
    def tgmem_accesses(self) -> tuple[TgmemAccess, ...]:
        return ()


@dataclass(frozen=True)
class MatmulAccumToTgFragment:
    config: MatmulConfig
    accumulator_suffix: str = ""
    emit_tg_coords: bool = True
    name: str = "matmul_accum_to_tg"
    kind: str = "store"

    def render(self, ctx: CodegenContext) -> str:
        t = self.config.tile
        Ct, suf = self.config.c_tile_name, self.accumulator_suffix
        return "\n".join(
            f"{Ct}[{t.row_of(i)}][{t.col_of(j)}] = acc{suf}[{i}][{j}];"
            for i in range(t.tm) for j in range(t.tn)
        )

    @property
    def tgmem_accesses(self) -> tuple[TgmemAccess, ...]:
        t = self.config.tile
        return (TgmemAccess(self.config.c_tile_name, "write", t.tile_M * (t.tile_N + t.c_pad),
                            (t.tile_M, t.tile_N + t.c_pad)),)


@dataclass(frozen=True)
class MatmulTgToDevFragment:
    config: MatmulConfig
    name: str = "matmul_tg_to_dev"
    kind: str = "store"

    def render(self, ctx: CodegenContext) -> str:
        from metellus_b200.memory.memory import TgStoreFragment

        t = self.config.tile
        return TgStoreFragment(
            name="store_C_tile", src_name=self.config.c_tile_name, dst_name=self.config.c_buffer_name,
            dst_row_stride=self.config.N_dim_var, row_start=f"tg.y * {t.tile_M}u",
            col_start=f"tg.x * {t.tile_N}u", tile_shape=(t.tile_M, t.tile_N),
            num_threads=t.num_threads, row_limit=self.config.M_dim_var,
            col_limit=self.config.N_dim_var, dst_col_stride=self.config.c_col_stride,
        ).render(ctx)

    @property
    def tgmem_accesses(self) -> tuple[TgmemAccess, ...]:
        t = self.config.tile
        return (TgmemAccess(self.config.c_tile_name, "read", t.tile_M * (t.tile_N + t.c_pad),
                            (t.tile_M, t.tile_N + t.c_pad)),)
