"""Elementwise strategies: STANDALONE_ELEMENTWISE, ELEMENTWISE_CHAIN (reference:
assembly/elementwise.py:17-128) and the B200 ELEMENTWISE_DAG.

All three render the same streaming kernel. The reference stages 16x16 tiles through
threadgroup memory; an elementwise op has no data reuse, so on B200 the kernel keeps
values in registers and streams HBM directly:

* grid-stride loop over the flat element space, ``U`` 128-bit vectors per thread per
  iteration, all loads issued before any arithmetic (memory-level parallelism);
* each distinct (buffer, strides, broadcast) operand is loaded once per element even
  when several ops read it (multi-root DAG: x feeds three chains in config C2);
* every tensor on the vertex boundary is written, so a DAG may have several
  materialised outputs;
* grid = SM count x resident blocks per SM (persistent), so the launch fills the 148
  SMs exactly once.

The vector path needs the inner extent to be a multiple of 4 (a vector never crosses a
row); otherwise the same kernel runs one element per step.
"""

from __future__ import annotations

from dataclasses import dataclass

from metellus_b200.compute.elementwise import BroadcastSpec, elementwise_expression
from metellus_b200.compute.fragments import CodegenContext, TgmemAccess
from metellus_b200.orchestrator.assembly.decision import DecisionView
from metellus_b200.orchestrator.assembly.expressions import scalar_literal, substitute, wrap_bool
from metellus_b200.orchestrator.assembly.extras import param_decl, pname
from metellus_b200.orchestrator.ir import ElementwiseOp, Scalar, Tensor
from metellus_b200.orchestrator.kernel_group import KernelGroup
from metellus_b200.runtime.program import Kernel

SM_COUNT = 148
EW_THREADS = 256
EW_BLOCKS_PER_SM = 8
EW_UNROLL = 2


def _canon_shape(t: Tensor) -> tuple[int, int, int]:
    """(batch, rows, cols) of a primary; a 1-D (M,) tensor is (1, M, 1)."""
    s = t.shape
    if len(s) == 3:
        return s
    if len(s) == 2:
        return (1, s[0], s[1])
    if len(s) == 1:
        return (1, s[0], 1)
    return (1, 1, 1)


def _strides3(t: Tensor) -> tuple[int, int, int]:
    """(batch, row, col) element strides of a tensor read in a (B, M, N) space."""
    if len(t.shape) == 3:
        return (t.batch_stride, t.row_stride, t.col_stride)
    if len(t.shape) == 2:
        return (0, t.row_stride, t.col_stride)
    if len(t.shape) == 1:
        return (0, t.row_stride, 0)
    return (0, 0, 0)


@dataclass(frozen=True)
class OperandRead:
    """One distinct external read: storage key, broadcast mode and strides."""

    key: str
    mode: BroadcastSpec
    strides: tuple[int, int, int]

    @property
    def var(self) -> str:
        s = "_".join(str(x) for x in self.strides).replace("-", "m")
        return f"in_{pname(self.key)}_{self.mode.value}_{s}"

    @property
    def ptr(self) -> str:
        return pname(self.key)


def external_reads(ops: tuple[ElementwiseOp, ...]) -> tuple[list[OperandRead], set[str]]:
    """Distinct external operand reads of an elementwise op set, in first-use order."""
    produced = {op.out.name for op in ops}
    reads: list[OperandRead] = []
    seen: set[OperandRead] = set()
    for op in ops:
        modes = (BroadcastSpec.NONE, op.y_broadcast, op.cond_broadcast)
        for k, o in enumerate(op.operands):
            if isinstance(o, Tensor) and o.name not in produced:
                r = OperandRead(o.buffer_key, modes[k], _strides3(o))
                if r not in seen:
                    seen.add(r)
                    reads.append(r)
    return reads, produced


def op_value_lines(ops: tuple[ElementwiseOp, ...], read_expr, lane: str = "") -> tuple[list[str], dict[str, str]]:
    """Per-element C++ statements evaluating ``ops`` in order. ``read_expr(op, k)``
    returns the expression for an external operand ``k`` of ``op``. Values are named
    ``v_<tensor>`` + ``lane`` suffix."""
    values: dict[str, str] = {}
    lines: list[str] = []
    for op in ops:
        subs = {}
        for k, key in enumerate(("x", "y", "cond")):
            if k >= len(op.operands):
                break
            o = op.operands[k]
            if isinstance(o, Scalar):
                subs[key] = f"({scalar_literal(o.value)})"
            elif o.name in values:
                subs[key] = f"({values[o.name]})"
            else:
                subs[key] = f"({read_expr(op, k)})"
        var = f"v{pname(op.out.name)}{lane}"
        lines.append(f"const float {var} = {wrap_bool(op.op, substitute(elementwise_expression(op.op), **subs))};")
        values[op.out.name] = var
    return lines, values


@dataclass(frozen=True)
class StreamingElementwiseFragment:
    """The whole streaming loop of an elementwise vertex (one fragment: the loop body
    is generated together because vector lanes share address arithmetic)."""

    ops: tuple[ElementwiseOp, ...]
    outputs: tuple[str, ...]
    shape: tuple[int, int, int]
    vector: bool
    unroll: int
    name: str = "streaming_elementwise"
    kind: str = "compute"

    @property
    def tgmem_accesses(self) -> tuple[TgmemAccess, ...]:
        return ()

    def render(self, ctx: CodegenContext) -> str:
        B, M, N = self.shape
        total = B * M * N
        NT = ctx.num_threads
        U = self.unroll
        reads, _ = external_reads(self.ops)
        out_keys = [op.out.buffer_key for op in self.ops if op.out.name in self.outputs]
        W = 4 if self.vector else 1
        nvec = total // W
        L = []
        L.append(f"for (size_t base = (size_t)blockIdx.x * {NT * U}u + threadIdx.x; base < {nvec}ull; "
                 f"base += (size_t)gridDim.x * {NT * U}u) {{")
        # Phase 1: coordinates and all loads.
        for u in range(U):
            L.append(f"  const size_t i{u} = base + {u * NT}u; const bool ok{u} = i{u} < {nvec}ull;")
            L.append(f"  const size_t e{u} = i{u} * {W}ull;")
            L.append(f"  const unsigned c{u} = (unsigned)(e{u} % {N}ull);")
            L.append(f"  const size_t rr{u} = e{u} / {N}ull;")
            L.append(f"  const unsigned r{u} = (unsigned)(rr{u} % {M}ull); const size_t b{u} = rr{u} / {M}ull;")
            for rd in reads:
                bs, rs, cs = rd.strides
                base_off = f"b{u} * {bs}ull" if bs else "0ull"
                v = f"{rd.var}_{u}"
                if rd.mode is BroadcastSpec.SCALAR:
                    L.append(f"  const float {v} = ok{u} ? mt_ldg({rd.ptr} + {base_off}) : 0.0f;")
                    continue
                if rd.mode is BroadcastSpec.COL or (rd.mode is BroadcastSpec.NONE and N == 1 and cs == 0):
                    L.append(f"  const float {v} = ok{u} ? mt_ldg({rd.ptr} + {base_off} + (size_t)r{u} * {rs}ll) : 0.0f;")
                    continue
                if rd.mode is BroadcastSpec.ROW:
                    if self.vector and cs == 1:
                        L.append(f"  float4 {v} = make_float4(0.f, 0.f, 0.f, 0.f); if (ok{u}) {v} = mt_ldg4({rd.ptr} + {base_off} + c{u});")
                    else:
                        self._lanes(L, v, W, u, rd.ptr, f"{base_off} + (size_t)(c{u} + LANE) * {cs}ll", cached=True)
                    continue
                # full-shape operand
                contiguous = (cs == 1 and rs == N and (bs == M * N or B == 1))
                if contiguous:
                    if self.vector:
                        L.append(f"  float4 {v} = make_float4(0.f, 0.f, 0.f, 0.f); if (ok{u}) {v} = mt_ld_stream4({rd.ptr} + e{u});")
                    else:
                        L.append(f"  const float {v} = ok{u} ? mt_ld_stream({rd.ptr} + e{u}) : 0.0f;")
                else:
                    self._lanes(L, v, W, u, rd.ptr,
                                f"{base_off} + (size_t)r{u} * {rs}ll + (size_t)(c{u} + LANE) * {cs}ll", cached=False)
        # Phase 2: arithmetic + stores.
        for u in range(U):
            L.append(f"  if (ok{u}) {{")
            lane_vals: list[dict[str, str]] = []
            for l in range(W):
                def rexpr(op, k, u=u, l=l):
                    o = op.operands[k]
                    mode = (BroadcastSpec.NONE, op.y_broadcast, op.cond_broadcast)[k]
                    rd = OperandRead(o.buffer_key, mode, _strides3(o))
                    v = f"{rd.var}_{u}"
                    if rd.mode is BroadcastSpec.SCALAR or rd.mode is BroadcastSpec.COL or \
                            (rd.mode is BroadcastSpec.NONE and N == 1 and rd.strides[2] == 0):
                        return v
                    return f"{v}.{'xyzw'[l]}" if W == 4 else v
                lines, vals = op_value_lines(self.ops, rexpr, lane=f"_{u}_{l}")
                L += ["    " + s for s in lines]
                lane_vals.append(vals)
            for op in self.ops:
                if op.out.name not in self.outputs:
                    continue
                key = pname(op.out.buffer_key)
                if W == 4:
                    comps = ", ".join(lane_vals[l][op.out.name] for l in range(4))
                    L.append(f"    mt_st_stream4({key} + e{u}, make_float4({comps}));")
                else:
                    L.append(f"    mt_st_stream({key} + e{u}, {lane_vals[0][op.out.name]});")
            L.append("  }")
        L.append("}")
        return "\n".join(L)

    @staticmethod
    def _lanes(L: list[str], v: str, W: int, u: int, key: str, off_tpl: str, cached: bool) -> None:
        ld = "mt_ldg" if cached else "mt_ld_stream"
        if W == 1:
            L.append(f"  const float {v} = ok{u} ? {ld}({key} + {off_tpl.replace('LANE', '0u')}) : 0.0f;")
            return
        L.append(f"  float4 {v} = make_float4(0.f, 0.f, 0.f, 0.f);")
        L.append(f"  if (ok{u}) {{ {v}.x = {ld}({key} + {off_tpl.replace('LANE', '0u')}); "
                 f"{v}.y = {ld}({key} + {off_tpl.replace('LANE', '1u')}); "
                 f"{v}.z = {ld}({key} + {off_tpl.replace('LANE', '2u')}); "
                 f"{v}.w = {ld}({key} + {off_tpl.replace('LANE', '3u')}); }}")


def assemble_elementwise(decision: DecisionView, function_name: str | None) -> KernelGroup:
    chain = decision.chain_only
    assert chain, "elementwise decision must carry ops"
    primary = chain[0].operands[0]
    assert isinstance(primary, Tensor)
    shape = _canon_shape(chain[0].out)
    B, M, N = shape
    outputs = decision.outputs or (chain[-1].out.name,)
    # A chain always materialises its tail (reference: assembly/elementwise.py:497).
    if chain[-1].out.name not in outputs:
        outputs = tuple(outputs) + (chain[-1].out.name,)
    reads, _ = external_reads(chain)
    # Binding order: primary, final output, then extras (reference slot order), then
    # any further outputs of a DAG.
    final_key = chain[-1].out.buffer_key
    in_keys: list[str] = [primary.buffer_key]
    for rd in reads:
        if rd.key not in in_keys:
            in_keys.append(rd.key)
    out_keys = [op.out.buffer_key for op in chain if op.out.name in outputs and op.out.buffer_key != final_key]
    bindings = (in_keys[0], final_key, *in_keys[1:], *out_keys)
    writable = {final_key, *out_keys}
    params = tuple(param_decl(k, writable=k in writable) for k in bindings)
    total = B * M * N
    vector = N % 4 == 0 and total % 4 == 0
    nvec = total // (4 if vector else 1)
    blocks = max(1, min(-(-nvec // (EW_THREADS * EW_UNROLL)), SM_COUNT * EW_BLOCKS_PER_SM))
    frag = StreamingElementwiseFragment(ops=chain, outputs=tuple(outputs), shape=shape, vector=vector,
                                        unroll=EW_UNROLL)
    fn = function_name or f"elementwise_{chain[-1].out.name}_fused"
    ctx = CodegenContext(function_name=fn, buffers=params, dims=("M", "N"), tg_x=EW_THREADS, tg_y=1)
    return KernelGroup(
        kernel=Kernel(fragments=(frag,), ctx=ctx),
        bindings=bindings,
        dims=(B * M, N),
        grid=(blocks, 1, 1),
        threads=(EW_THREADS, 1, 1),
        ops=decision.ops,
        strategy=decision.strategy,
    )
