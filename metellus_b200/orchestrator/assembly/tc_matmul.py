"""tcgen05 / TMEM 3xTF32 tensor-core pipe for matmul groups (B200).

Every matmul strategy (standalone, register or shared-tile epilogue, elementwise
prologue) and the two-anchor strategies (multi-producer convergent, diamond, dual GEMM)
lower to one warp-specialised kernel from csrc/include/mt_tc.cuh:

* a TMA warp (128-byte swizzle) streams 128 x 32 A tiles and the B tiles of every
  anchor into a raw ring of shared-memory stages;
* six converter warps apply the prologue chain (read at the element's global
  (row, k)) and split each fp32 value into tf32 hi / lo: A rows into tensor memory,
  B tiles into a converted ring in shared memory;
* two threads (even / odd k-tiles) issue ``tcgen05.mma.kind::tf32`` for hi*lo + lo*hi +
  hi*hi into a fresh TMEM accumulator per 32-deep k-tile (one issuer alone leaves the
  tensor pipe idle while it waits on barriers);
* eight accumulator warps add each finished k-tile into fp32 registers and run the
  epilogue (the fused elementwise chain, or the two-anchor merge / DAG) at each
  element's global (row, col).

Tile shapes: ``mt_gemm_3xtf32_pair`` (256 x 128 per two-CTA cluster, ``cta_group::2``)
when the output has enough such tiles to fill the SMs; otherwise ``mt_gemm_3xtf32``
with 128 x BN tiles on one CTA, and split-K over a two-CTA cluster when even those are
too few. Shapes the tensor maps cannot describe (batched operands, unaligned strides,
an MN-major operand whose extent is not a multiple of 32) or tiny problems stay on the
SIMT FFMA pipe. ``METELLUS_TC=0`` forces FFMA; ``METELLUS_TC_PAIR=0`` disables the pair
tiles.
"""

from __future__ import annotations

import os
from dataclasses import dataclass

from metellus_b200.compute.device_lib import header
from metellus_b200.compute.elementwise import BroadcastSpec, elementwise_expression
from metellus_b200.compute.fragments import CodegenContext, TgmemAccess
from metellus_b200.orchestrator.assembly.decision import DecisionView
from metellus_b200.orchestrator.assembly.expressions import (
    chain_value_transform,
    scalar_literal,
    substitute,
    wrap_bool,
)
from metellus_b200.orchestrator.assembly import pipe_table
from metellus_b200.orchestrator.assembly.extras import Extras, param_decl, pname
from metellus_b200.orchestrator.ir import ElementwiseOp, MatmulOp, Scalar, Tensor
from metellus_b200.orchestrator.kernel_group import STATUS_BYTES, STATUS_KEY, FusionStrategy, KernelGroup
from metellus_b200.runtime.program import Kernel, TmapSpec

SM_COUNT = 148
SMEM_BUDGET = 200 * 1024
MIN_VOLUME = 64 * 64 * 64


def tc_enabled() -> bool:
    return os.environ.get("METELLUS_TC", "1") != "0"


def _a_layout(t: Tensor) -> str | None:
    """'k' (K contiguous), 'mn' (M contiguous) or None when TMA cannot describe it."""
    if len(t.shape) != 2:
        return None
    M, K = t.shape
    if t.col_stride == 1 and (t.row_stride * 4) % 16 == 0 and (M == 1 or t.row_stride >= K):
        return "k"
    return None


def _b_layout(t: Tensor) -> str | None:
    if len(t.shape) != 2:
        return None
    K, N = t.shape
    if t.col_stride == 1 and (t.row_stride * 4) % 16 == 0 and N % 32 == 0 and t.row_stride >= N:
        return "mn"
    if t.row_stride == 1 and (t.col_stride * 4) % 16 == 0 and t.col_stride >= K:
        return "k"
    return None


def _tmap(buf_index: int, t: Tensor, layout: str, outer_box: int) -> TmapSpec:
    """Tensor map for a 128-byte-swizzled operand tile of 32 k-columns.

    K-major: 2-D {K, rows} box {32, outer_box}. MN-major: 3-D {32, K, rows/32} box
    {32, 32, outer_box/32} — 32-wide chunks along M/N land 4 KB apart."""
    R, K = (t.shape[0], t.shape[1])
    if layout == "k":
        if t.col_stride == 1:  # A-like: rows along dim 0
            rows, ld = t.shape[0], t.row_stride
            kdim = t.shape[1]
        else:  # B stored K-contiguous: rows are n, ld = col_stride
            rows, ld = t.shape[1], t.col_stride
            kdim = t.shape[0]
        return TmapSpec(buf_index, (kdim, rows), (ld * 4,), (32, outer_box))
    # MN-major
    if t.row_stride == 1:  # A col-major: contiguous along M, ld = col_stride
        rows, ld, kdim = t.shape[0], t.col_stride, t.shape[1]
    else:  # B row-major: contiguous along N, ld = row_stride
        rows, ld, kdim = t.shape[1], t.row_stride, t.shape[0]
    # 128-byte swizzle on 32-byte atoms: the layout tcgen05 reads tf32 MN-major operands in
    return TmapSpec(buf_index, (32, kdim, rows // 32), (ld * 4, 128), (32, 32, outer_box // 32), swizzle=4)


def _raw_bytes(bn: int, nb: int) -> int:
    """A raw-ring stage: the TMA targets A and B of every anchor."""
    return 128 * 32 * 4 + nb * bn * 32 * 4


def _conv_bytes(bn: int, nb: int) -> int:
    """A converted-ring stage: B hi + B lo of every anchor (A's split lives in tensor
    memory)."""
    return 2 * nb * bn * 32 * 4


def _pick_tile(M: int, N: int, nb: int, b_mn: bool = True, K: int = 0) -> tuple[int, int, int]:
    """(BN, stages, split-K): the widest N tile that still gives ~one CTA per SM; as
    many stages (each raw + converted ring gets `stages` entries) as fit the
    shared-memory budget and tensor memory (512 columns: two accumulator chunks of
    nb * BN columns, plus 64 columns of A hi / lo per converted stage). A k-tile costs
    about the same time at BN = 64 as at 128 (the A split and the pipeline hand-offs
    dominate), so an output with too few 128-wide tiles to fill the SMs keeps BN = 128
    and splits K over a two-CTA cluster instead of halving BN (C = 1024^3: 64 tiles ->
    128 CTAs of 16 k-tiles each)."""
    tiles_m = -(-M // 128)
    tiles128 = tiles_m * -(-N // 128)
    splitk = 1
    if nb == 1 and tiles128 >= SM_COUNT * 0.8:
        bn = 128
    elif nb == 1 and 2 * tiles128 <= SM_COUNT and -(-K // 32) >= 16:
        bn, splitk = 128, 2
    else:
        bn = 64
    return bn, _stages(bn, nb), splitk


def _stages(bn: int, nb: int) -> int:
    tmem_stages = (512 - 2 * nb * bn) // 64
    return max(2, min(4, tmem_stages, SMEM_BUDGET // (_raw_bytes(bn, nb) + _conv_bytes(bn, nb))))


def _choose_tiling(M: int, N: int, K: int, nb: int, b_mn: bool) -> tuple[int, int, int, tuple | None]:
    """(BN, stages, split-K, pair parameters or None) of a tcgen05 matmul group: the
    measured pick of ``pipe_table`` where it covers the shape, else the heuristics
    (``_pick_pair``, then ``_pick_tile``). Split-K exists for one anchor only."""
    bn, stages, splitk = _pick_tile(M, N, nb, b_mn, K)
    pair = _pick_pair(M, N, nb)
    pick = pipe_table.lookup(M, N, K, nb)
    if pick is not None and pick.variant == "pair":
        pair = _pick_pair(M, N, nb, force=True)
    elif pick is not None and pick.variant in ("one", "splitk"):
        pair = None
        if pick.variant == "splitk" and nb == 1 and -(-K // 32) >= 2:
            bn, splitk = 128, 2
        else:
            splitk = 1
        stages = _stages(bn, nb)
    if pair is not None:
        bn, splitk = pair[0], 1
    return bn, stages, splitk, pair


def _smem_bytes(bn: int, stages: int, nb: int, b_mn: bool = True) -> int:
    return stages * (_raw_bytes(bn, nb) + _conv_bytes(bn, nb)) + (4 * stages + 6) * 8 + 16 + 1024


# CTA-pair (cta_group::2) tiles: 256 x 128 per two-CTA cluster, 64 B rows per CTA.
PAIR_RAW_BYTES = 128 * 32 * 4 + 64 * 32 * 4     # A + this CTA's half of B
PAIR_CONV_BYTES = 2 * 64 * 32 * 4               # B hi + lo
# Accumulation (split accumulators): one issuing thread accumulates hi*hi into a chunk
# buffer of 128 columns that the accumulator warps promote into fp32 registers every
# PAIR_CHUNK k-tiles; a second thread accumulates the small products hi*lo + lo*hi of
# the whole K into a buffer of their own, added once at the end.
PAIR_SACC = int(os.environ.get("METELLUS_TC_SACC", "1"))
PAIR_NACC = 1 if PAIR_SACC else 2   # chunk buffers of 128 columns
PAIR_CHUNK = int(os.environ.get("METELLUS_TC_CHUNK", "3")) if PAIR_SACC else 1   # k-tiles per promotion
PAIR_ISSUERS = 2    # MMA-issuing threads (warps 1 and 0); 1 measured 7-10 % slower
PAIR_THREADS = 544  # 17 warps (both GEMM kernels): the 17th issues the TMA loads
# tensor memory: accumulator buffers + 64 columns of A (hi, lo) per converted stage
PAIR_CSTAGES = (512 - 128 * (PAIR_NACC + PAIR_SACC)) // 64


def pair_enabled() -> bool:
    return os.environ.get("METELLUS_TC_PAIR", "1") != "0"


def _pick_pair(M: int, N: int, nb: int, force: bool = False) -> tuple[int, int, int] | None:
    """(BN, raw stages, converted stages) of a CTA-pair tile, or None when the output
    has too few 256 x 128 pair tiles to fill the SMs (about one pair per two SMs)
    and ``force`` is not set."""
    if not pair_enabled():
        return None
    bn = 128 // nb
    pairs = -(-M // 256) * -(-N // bn)
    if pairs < 0.8 * SM_COUNT / 2 and not force:
        return None
    cst = PAIR_CSTAGES
    rst = max(2, min(6, (SMEM_BUDGET - cst * PAIR_CONV_BYTES) // PAIR_RAW_BYTES))
    return bn, rst, cst


def _pair_group_m(K: int) -> int:
    """M tiles (of 256 rows) per group of the pair kernel's tile order. Consecutive
    clusters walk all N tiles of one group, so each group's A rows stay in L2 while
    the whole B panel streams past, and B is read once per group. Measured on the C5
    GEMMs (DRAM bytes per launch, ncu): the dual GEMM (K = 2048, 2 MB of A per M
    tile) reads 4.36 / 2.27 / 1.21 / 0.68 / 2.48 GB with groups of 2 / 4 / 8 / 16 / 32
    (32 overflows L2); the down-projection (K = 8192, 8 MB per M tile) 1.81 / 2.01 /
    2.09 / 2.73 / 5.76 GB. So about 32 MB of A per group, and at least 2 tiles."""
    a_tile = 256 * K * 4
    return 16 if (32 << 20) // a_tile >= 16 else 2


def _pair_smem_bytes(rst: int, cst: int) -> int:
    return rst * PAIR_RAW_BYTES + cst * PAIR_CONV_BYTES + (2 * rst + 2 * cst + 2 * PAIR_NACC + 3) * 8 + 16 + 1024


def _read(t: Tensor, mode: BroadcastSpec, row: str, col: str) -> str:
    p = pname(t.buffer_key)
    rs, cs = t.row_stride, t.col_stride
    if len(t.matrix_shape) == 1:
        return f"{p}[(size_t)({row}) * {rs}ll]"
    if mode is BroadcastSpec.SCALAR:
        return f"{p}[0]"
    if mode is BroadcastSpec.ROW:
        return f"__ldg({p} + (size_t)({col}) * {cs}ll)"
    if mode is BroadcastSpec.COL:
        return f"{p}[(size_t)({row}) * {rs}ll]"
    return f"{p}[(size_t)({row}) * {rs}ll + (size_t)({col}) * {cs}ll]"


def epilogue_lines(ops: tuple[ElementwiseOp, ...], acc_names: dict[str, str], row: str, col: str,
                   suffix: str) -> tuple[list[str], dict[str, str]]:
    """Per-element statements of an epilogue op list; ``acc_names`` maps anchor
    outputs to accumulator expressions."""
    vals = dict(acc_names)
    lines = []
    for i, op in enumerate(ops):
        subs = {}
        modes = (BroadcastSpec.NONE, op.y_broadcast, op.cond_broadcast)
        for k, key in enumerate(("x", "y", "cond")[: len(op.operands)]):
            o = op.operands[k]
            if isinstance(o, Scalar):
                subs[key] = f"({scalar_literal(o.value)})"
            elif o.name in vals:
                subs[key] = f"({vals[o.name]})"
            else:
                subs[key] = f"({_read(o, modes[k], row, col)})"
        v = f"e{i}{suffix}"
        lines.append(f"const float {v} = {wrap_bool(op.op, substitute(elementwise_expression(op.op), **subs))};")
        vals[op.out.name] = v
    return lines, vals


@dataclass(frozen=True)
class TcGemmFragment:
    """The whole tcgen05 GEMM: lambdas for prologues / epilogue and the mainloop call."""

    bn: int
    stages: int
    a_mn: bool  # always False: A tiles are K-major
    b_mn: bool
    nb: int
    pro_a: str | None           # expression in (x, r, c) or None
    pro_b: str | None
    epi_body: str               # body of the per-(row, 32 columns) store lambda
    splitk: int = 1             # 2: two-CTA cluster per tile, K halves combined via DSMEM
    pair: tuple[int, int] | None = None  # (raw, converted) stages of a CTA-pair tile
    group_m: int = 8            # pair tiles: M tiles per group of the tile order
    name: str = "tc_gemm"
    kind: str = "compute"

    @property
    def arena_bytes(self) -> int:
        if self.pair is not None:
            return _pair_smem_bytes(*self.pair)
        return _smem_bytes(self.bn, self.stages, self.nb, self.b_mn)

    @property
    def tgmem_accesses(self) -> tuple[TgmemAccess, ...]:
        n = self.arena_bytes // 4
        return (TgmemAccess("tc_arena", "readwrite", n, (1, n)),)

    def render(self, ctx: CodegenContext) -> str:
        lines = []
        for side, expr in (("a", self.pro_a), ("b", self.pro_b)):
            if expr is None:
                lines.append(f"const mt_no_prologue pro_{side}{{}};")
            else:
                lines.append(f"auto pro_{side}_f = [=](float x, int r, int c) -> float {{ return {expr}; }};")
                lines.append(f"const mt_prologue<decltype(pro_{side}_f)> pro_{side}{{pro_{side}_f}};")
        lines.append(f"auto epi_f = [=](int row, int col0, float (&v)[{self.nb}][32]) {{\n{self.epi_body}\n}};")
        lines.append("const mt_epilogue<decltype(epi_f)> epi{epi_f};")
        tb1 = "&tm_b1" if self.nb > 1 else "&tm_b0"
        if self.pair is not None:
            rst, cst = self.pair
            # BAL: warps 2-3 split B while warps 4-7 split A (~1% faster)
            lines.append(
                f"mt_gemm_3xtf32_pair<{self.bn}, {rst}, {cst}, {str(self.b_mn).lower()}, {self.nb}, {PAIR_CHUNK}, "
                f"true, {PAIR_NACC}, {PAIR_ISSUERS}, {str(bool(PAIR_SACC)).lower()}, {self.group_m}>"
                f"(&tm_a, &tm_b0, {tb1}, (int)M, (int)N, (int)K, pro_a, pro_b, epi, g_status, tc_arena);")
            return "\n".join(lines)
        lines.append(
            f"mt_gemm_3xtf32<{self.bn}, {self.stages}, {self.stages}, {str(self.a_mn).lower()}, "
            f"{str(self.b_mn).lower()}, "
            f"{self.nb}, {self.splitk}>(&tm_a, &tm_b0, {tb1}, (int)M, (int)N, (int)K, pro_a, pro_b, epi, g_status, "
            "tc_arena);"
        )
        return "\n".join(lines)


def _store_lines(out_key: str, ldo: int, vals_for_j, N: int, need_col_check: bool) -> str:
    """Store the 32 columns [col0, col0 + 32) of ``row`` (float4 where possible)."""
    p = pname(out_key)
    body = ["if (row >= (int)M) return;"]
    if need_col_check or ldo % 4 != 0:
        body.append("#pragma unroll\nfor (int j = 0; j < 32; ++j) {")
        body.append(f"  if (col0 + j < (int)N) {p}[(size_t)row * {ldo}ull + col0 + j] = {vals_for_j('j')};")
        body.append("}")
    else:
        body.append("if (col0 >= (int)N) return;")
        body.append(f"float* dst = {p} + (size_t)row * {ldo}ull + col0;")
        body.append("#pragma unroll\nfor (int j = 0; j < 32; j += 4) {")
        body.append(f"  float4 o; o.x = {vals_for_j('j')}; o.y = {vals_for_j('j + 1')}; "
                    f"o.z = {vals_for_j('j + 2')}; o.w = {vals_for_j('j + 3')};")
        body.append("  *reinterpret_cast<float4*>(dst + j) = o;")
        body.append("}")
    return "\n".join(body)


def _epi_function(ops, acc_names: dict[str, str], out_key: str, final: str, N: int, ldo: int,
                  need_col_check: bool) -> str:
    """Epilogue lambda body: evaluates ``ops`` per element and stores ``final``."""
    # evaluate per element via a small inline function of j
    lines, vals = epilogue_lines(ops, acc_names, "row", "col0 + J", "")
    fn = ["auto elem = [&](int J) -> float {"] + ["  " + l for l in lines] + [f"  return {vals[final]};", "};"]
    body = "\n".join(fn) + "\n" + _store_lines(out_key, ldo, lambda j: f"elem({j})", N, need_col_check)
    return body


def _fits_cap(nbytes: int) -> bool:
    """The tensor-core tiles need ~200 KB of shared memory; under a smaller budget
    cap (e.g. the reference's 32 KB, used to reproduce its plans) the SIMT pipe is
    chosen instead."""
    from metellus_b200.orchestrator import fusion

    return nbytes <= fusion.TGMEM_CAP_BYTES


def _common_checks(a_src: Tensor, b_src: Tensor, M: int, N: int, K: int, nb: int = 1) -> tuple[str, str] | None:
    if not tc_enabled() or not _fits_cap(SMEM_BUDGET):
        return None
    pick = pipe_table.lookup(M, N, K, nb)
    if pick is not None and pick.variant == "ffma":
        return None
    if pick is None and M * N * K < MIN_VOLUME:
        return None
    la, lb = _a_layout(a_src), _b_layout(b_src)
    if la is None or lb is None:
        return None
    return la, lb


def try_assemble_tc_matmul(decision: DecisionView, function_name: str | None) -> KernelGroup | None:
    anchor = decision.anchor
    assert isinstance(anchor, MatmulOp)
    if len(anchor.out.shape) != 2:
        return None
    src_a = decision.prologue_a[0].operands[0] if decision.prologue_a else anchor.a
    src_b = decision.prologue_b[0].operands[0] if decision.prologue_b else anchor.b
    assert isinstance(src_a, Tensor) and isinstance(src_b, Tensor)
    M, K = anchor.a.shape
    N = anchor.b.shape[1]
    lay = _common_checks(src_a, src_b, M, N, K)
    if lay is None:
        return None
    la, lb = lay
    if decision.prologue_b and lb == "mn":
        return None  # prologue coordinates are only decoded for K-major B tiles
    final_out = decision.epilogue[-1].out if decision.epilogue else anchor.out
    out_key = final_out.buffer_key

    in_slots: dict[str, int] = {}
    for t in (src_a, src_b):
        if t.buffer_key not in in_slots:
            in_slots[t.buffer_key] = len(in_slots)
    out_slot = len(in_slots)
    base = out_slot + 1
    extras = Extras(base_slots_by_key={**in_slots, out_key: out_slot})
    pro_a = chain_value_transform(decision.prologue_a, row_var="r", col_var="c", extras=extras,
                                  base_slot=base)("x") if decision.prologue_a else None
    pro_b = chain_value_transform(decision.prologue_b, row_var="r", col_var="c", extras=extras,
                                  base_slot=base)("x") if decision.prologue_b else None
    for op in decision.epilogue:
        for o in op.inputs:
            if o.name not in {e.out.name for e in decision.epilogue} and o.name != anchor.out.name:
                extras.add_tensor(o, base)
    bn, stages, splitk, pair = _choose_tiling(M, N, K, 1, lb == "mn")
    need_col_check = N % 32 != 0
    epi = _epi_function(decision.epilogue, {anchor.out.name: "v[0][J]"}, out_key,
                        final_out.name, N, N, need_col_check)
    bindings = (*in_slots.keys(), out_key, *extras.bindings)
    params = tuple(param_decl(k, writable=(k == out_key)) for k in bindings) + ("int* g_status",)
    tmaps = (
        _tmap(bindings.index(src_a.buffer_key), src_a, la, 128),
        _tmap(bindings.index(src_b.buffer_key), src_b, lb, 64 if pair else bn),
    )
    frag = TcGemmFragment(bn=bn, stages=stages, a_mn=la == "mn", b_mn=lb == "mn", nb=1, pro_a=pro_a,
                          pro_b=pro_b, epi_body=epi, splitk=splitk, pair=pair[1:] if pair else None,
                          group_m=_pair_group_m(K))
    n_arena = frag.arena_bytes // 4
    fn = function_name or f"tc_matmul_{anchor.out.name}_fused"
    ctx = CodegenContext(
        function_name=fn, buffers=params, dims=("M", "K", "N"), tg_x=PAIR_THREADS, tg_y=1,
        threadgroup_decls=(f"smem float tc_arena[{n_arena}];",),
        helpers=(header("mt_tc.cuh"),),
        extra_params=("const __grid_constant__ mt_tmap tm_a", "const __grid_constant__ mt_tmap tm_b0"),
        min_blocks_per_sm=1,
    )
    return KernelGroup(
        kernel=Kernel(fragments=(frag,), ctx=ctx), bindings=bindings, dims=(M, K, N),
        grid=(2 * -(-N // bn), -(-M // 256), 1) if pair else (splitk * -(-N // bn), -(-M // 128), 1),
        threads=(PAIR_THREADS, 1, 1), ops=decision.ops,
        strategy=decision.strategy, pipe="tcgen05", tmaps=tmaps, scratch=((STATUS_KEY, STATUS_BYTES),),
        cluster_x=2 if pair else splitk,
    )


def dual_gemm_eligible(a0: MatmulOp, a1: MatmulOp) -> bool:
    """Whether two anchors sharing A can run as one tcgen05 kernel (2-D, same K and
    N, tensor-map-able operands with one B layout)."""
    if len(a0.out.shape) != 2 or a0.out.shape != a1.out.shape or a0.a.name != a1.a.name:
        return False
    M, K = a0.a.shape
    N = a0.b.shape[1]
    lay = _common_checks(a0.a, a0.b, M, N, K, 2)
    return lay is not None and _b_layout(a1.b) == lay[1]


def try_assemble_tc_multi_anchor(decision: DecisionView, function_name: str | None) -> KernelGroup | None:
    """Two anchors sharing A (diamond): one mainloop, two TMEM accumulators, the merge
    (or, for a dual-GEMM vertex, the whole elementwise DAG over both accumulators)
    applied in the epilogue. Other two-anchor shapes stay on the SIMT pipe."""
    if not decision.shared_a:
        return None
    a0, a1 = decision.anchors
    merge = decision.merge_elem
    epi_ops = decision.epilogue or (merge,)
    if len(a0.out.shape) != 2 or decision.prologues_b[0] or decision.prologues_b[1]:
        return None
    M, K = a0.a.shape
    N = a0.b.shape[1]
    if a1.a.shape[1] != K:
        return None
    lay = _common_checks(a0.a, a0.b, M, N, K, 2)
    if lay is None or _b_layout(a1.b) != lay[1]:
        return None
    la, lb = lay
    out_key = merge.out.buffer_key
    in_keys: list[str] = []
    for t in (a0.a, a0.b, a1.b):
        if t.buffer_key not in in_keys:
            in_keys.append(t.buffer_key)
    out_slot = len(in_keys)
    extras = Extras(base_slots_by_key={**{k: i for i, k in enumerate(in_keys)}, out_key: out_slot})
    inside = {a0.out.name, a1.out.name} | {op.out.name for op in epi_ops}
    for op in epi_ops:
        for o in op.inputs:
            if o.name not in inside:
                extras.add_tensor(o, out_slot + 1)
    bn, stages, _, pair = _choose_tiling(M, N, K, 2, lb == "mn")
    epi = _epi_function(tuple(epi_ops), {a0.out.name: "v[0][J]", a1.out.name: "v[1][J]"}, out_key,
                        merge.out.name, N, N, N % 32 != 0)
    bindings = (*in_keys, out_key, *extras.bindings)
    params = tuple(param_decl(k, writable=(k == out_key)) for k in bindings) + ("int* g_status",)
    tmaps = (
        _tmap(bindings.index(a0.a.buffer_key), a0.a, la, 128),
        _tmap(bindings.index(a0.b.buffer_key), a0.b, lb, 64 if pair else bn),
        _tmap(bindings.index(a1.b.buffer_key), a1.b, lb, 64 if pair else bn),
    )
    frag = TcGemmFragment(bn=bn, stages=stages, a_mn=la == "mn", b_mn=lb == "mn", nb=2, pro_a=None, pro_b=None,
                          epi_body=epi, pair=pair[1:] if pair else None, group_m=_pair_group_m(K))
    n_arena = frag.arena_bytes // 4
    fn = function_name or f"tc_diamond_{merge.out.name}_fused"
    ctx = CodegenContext(
        function_name=fn, buffers=params, dims=("M", "K", "N"), tg_x=PAIR_THREADS, tg_y=1,
        threadgroup_decls=(f"smem float tc_arena[{n_arena}];",),
        helpers=(header("mt_tc.cuh"),),
        extra_params=("const __grid_constant__ mt_tmap tm_a", "const __grid_constant__ mt_tmap tm_b0",
                      "const __grid_constant__ mt_tmap tm_b1"),
        min_blocks_per_sm=1,
    )
    return KernelGroup(
        kernel=Kernel(fragments=(frag,), ctx=ctx), bindings=bindings, dims=(M, K, N),
        grid=(2 * -(-N // bn), -(-M // 256), 1) if pair else (-(-N // bn), -(-M // 128), 1),
        threads=(PAIR_THREADS, 1, 1), ops=decision.ops,
        strategy=decision.strategy, pipe="tcgen05", tmaps=tmaps, scratch=((STATUS_KEY, STATUS_BYTES),),
        cluster_x=2 if pair else 1,
    )
