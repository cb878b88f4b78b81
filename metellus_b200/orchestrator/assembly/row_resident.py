"""ROW_RESIDENT strategy (B200): reductions plus the elementwise ops around them, over
one row space, in one kernel that keeps each row in registers.

The reference lowers a row softmax to four kernels (max-reduce, [sub, exp],
sum-reduce, div) and a layernorm to four as well, each re-reading the full matrix
from memory. Here one CTA owns a row at a time (grid-stride over rows, grid sized to
the SMs): every external full-row operand is loaded once with 128-bit loads into
registers, the op list runs in program order — row-vector ops lane by lane, each
reduction as a thread-local fold plus one warp-shuffle / shared-memory block
all-reduce, per-row scalar ops once — and every tensor on the vertex boundary is
stored once. HBM traffic is the algorithmic minimum: one read of each input row and
one write of each output row.

Value kinds inside the kernel: *vector* (one value per element of the row: a
(rows, K) tensor), *scalar* (one value per row: a reduction output, a (M,) / (M, 1)
tensor or a view between the two), *column* (an external (1, K) row-broadcast
operand, same for every row).
"""

from __future__ import annotations

from dataclasses import dataclass

from metellus_b200.compute.elementwise import BroadcastSpec, elementwise_expression
from metellus_b200.compute.fragments import CodegenContext, TgmemAccess
from metellus_b200.compute.reduction import reduction_combiner
from metellus_b200.orchestrator.assembly.decision import DecisionView
from metellus_b200.orchestrator.assembly.expressions import scalar_literal, substitute, wrap_bool
from metellus_b200.orchestrator.assembly.extras import param_decl, pname
from metellus_b200.orchestrator.ir import ElementwiseOp, Op, ReductionOp, Scalar, Tensor
from metellus_b200.orchestrator.kernel_group import KernelGroup
from metellus_b200.runtime.program import Kernel

SM_COUNT = 148


def _is_vector_tensor(t: Tensor) -> bool:
    s = t.matrix_shape
    return len(s) == 2 and s[1] != 1


def _rows_of(t: Tensor) -> tuple[int, int]:
    """(batch, rows per batch) of a tensor in the row space."""
    s = t.shape
    if len(s) == 3:
        return s[0], s[1]
    return 1, s[0]


def _same_layout(view: Tensor, owner: Tensor) -> bool:
    """Whether a view addresses its owner's elements at the owner's own (row, col):
    same shape and strides. A transposed view of a square matrix has the owner's shape
    but swapped strides, so it is not row local."""
    return (view.shape == owner.shape and view.row_stride == owner.row_stride
            and view.col_stride == owner.col_stride
            and (len(view.shape) != 3 or view.batch_stride == owner.batch_stride))


def row_program_check(ops: tuple[Op, ...]) -> str | None:
    """Why ``ops`` cannot run row-resident, or None when they can."""
    produced = {op.out.name: op for op in ops}
    kinds: dict[str, str] = {}
    for op in ops:
        if isinstance(op, ReductionOp):
            src = op.input
            k = kinds.get(src.name) or (kinds.get(src.buffer_key) if src.buffer_key in produced else None)
            if src.name in produced or src.buffer_key in produced:
                if k != "vector" or (src.name not in produced and not _same_layout(src, produced[src.buffer_key].out)):
                    return f"reduction {op.out.name!r} reads a non row-local view"
            kinds[op.out.name] = "scalar"
        elif isinstance(op, ElementwiseOp):
            vec = _is_vector_tensor(op.out)
            for o in op.operands:
                if not isinstance(o, Tensor):
                    continue
                owner = o.name if o.name in produced else (o.buffer_key if o.buffer_key in produced else None)
                if owner is None:
                    continue
                ko = kinds[owner]
                if ko == "vector" and (o.name != owner and not _same_layout(o, produced[owner].out)):
                    return f"{op.out.name!r} reads a reshaped view of row vector {owner!r}"
                if ko == "scalar" and _is_vector_tensor(o):
                    return f"{op.out.name!r} reads per-row scalar {owner!r} as a full row"
                if ko == "scalar" and vec and o is op.operands[0]:
                    return f"{op.out.name!r} has a per-row scalar primary"
            kinds[op.out.name] = "vector" if vec else "scalar"
        else:
            return f"{type(op).__name__} cannot run row-resident"
    return None


@dataclass(frozen=True)
class RowResidentFragment:
    ops: tuple[Op, ...]
    outputs: tuple[str, ...]
    rows: int          # total rows (batch * rows per batch)
    rows_per_batch: int
    cols: int
    width: int         # 4 (float4 chunks) or 1
    chunks: int        # chunks per thread
    name: str = "row_resident"
    kind: str = "compute"

    @property
    def tgmem_accesses(self) -> tuple[TgmemAccess, ...]:
        return (TgmemAccess("red_scratch", "readwrite", 33, (1, 33)),)

    def render(self, ctx: CodegenContext) -> str:
        NT = ctx.num_threads
        W, P, K, R, Mb = self.width, self.chunks, self.cols, self.rows, self.rows_per_batch
        produced = {op.out.name: op for op in self.ops}
        L: list[str] = []
        L.append(f"for (unsigned row = blockIdx.x; row < {R}u; row += gridDim.x) {{")
        L.append(f"  const unsigned bidx = row / {Mb}u, mrow = row % {Mb}u;")
        # chunk validity
        for p in range(P):
            L.append(f"  const unsigned col{p} = ({p}u * {NT}u + threadIdx.x) * {W}u; const bool ok{p} = col{p} < {K}u;")
        kinds: dict[str, str] = {}
        vals: dict[str, str] = {}        # value name -> C var (vector: array base name)
        loaded: dict[tuple, str] = {}
        # All external loads are hoisted to the top of the row body (issued before any
        # arithmetic); ``LD`` collects them while the op walk fills ``L``.
        head = L
        LD: list[str] = []
        L = []

        def owner_of(t: Tensor) -> str | None:
            if t.name in produced:
                return t.name
            if t.buffer_key in produced:
                return t.buffer_key
            return None

        def ext_vec(t: Tensor) -> str:
            key = ("vec", t.buffer_key, t.row_stride, t.col_stride, t.batch_stride)
            if key in loaded:
                return loaded[key]
            var = f"x{len(loaded)}"
            loaded[key] = var
            ptr = pname(t.buffer_key)
            bs = t.batch_stride if len(t.shape) == 3 else 0
            base = f"(size_t)bidx * {bs}ull + (size_t)mrow * {t.row_stride}ll"
            LD.append(f"  float {var}[{P}][{W}];")
            for p in range(P):
                if W == 4 and t.col_stride == 1:
                    LD.append(f"  {{ float4 t4 = make_float4(0.f, 0.f, 0.f, 0.f); if (ok{p}) t4 = mt_ld_stream4({ptr} + {base} + col{p});"
                             f" {var}[{p}][0] = t4.x; {var}[{p}][1] = t4.y; {var}[{p}][2] = t4.z; {var}[{p}][3] = t4.w; }}")
                else:
                    for l in range(W):
                        LD.append(f"  {var}[{p}][{l}] = (col{p} + {l}u < {K}u) ? mt_ld_stream({ptr} + {base} + (size_t)(col{p} + {l}u) * {t.col_stride}ll) : 0.0f;")
            return var

        def ext_col(t: Tensor) -> str:
            """(1, K) row-broadcast operand: same for every row."""
            key = ("col", t.buffer_key, t.col_stride)
            if key in loaded:
                return loaded[key]
            var = f"x{len(loaded)}"
            loaded[key] = var
            ptr = pname(t.buffer_key)
            bs = t.batch_stride if len(t.shape) == 3 else 0
            LD.append(f"  float {var}[{P}][{W}];")
            for p in range(P):
                for l in range(W):
                    LD.append(f"  {var}[{p}][{l}] = (col{p} + {l}u < {K}u) ? mt_ldg({ptr} + (size_t)bidx * {bs}ull + (size_t)(col{p} + {l}u) * {t.col_stride}ll) : 0.0f;")
            return var

        def ext_scalar(t: Tensor, mode: BroadcastSpec) -> str:
            key = ("scal", t.buffer_key, t.row_stride, t.col_stride, mode.value)
            if key in loaded:
                return loaded[key]
            var = f"x{len(loaded)}"
            loaded[key] = var
            ptr = pname(t.buffer_key)
            bs = t.batch_stride if len(t.shape) == 3 else 0
            if mode is BroadcastSpec.SCALAR:
                LD.append(f"  const float {var} = mt_ldg({ptr} + (size_t)bidx * {bs}ull);")
            else:
                rs = t.row_stride
                LD.append(f"  const float {var} = mt_ldg({ptr} + (size_t)bidx * {bs}ull + (size_t)mrow * {rs}ll);")
            return var

        def ref(o, mode: BroadcastSpec, want_vector: bool):
            """Return (kind, expr-or-var) of an operand."""
            if isinstance(o, Scalar):
                return ("lit", scalar_literal(o.value))
            own = owner_of(o)
            if own is not None:
                return (kinds[own], vals[own])
            if _is_vector_tensor(o):
                if mode is BroadcastSpec.ROW:
                    return ("vector", ext_col(o))
                return ("vector", ext_vec(o))
            if mode is BroadcastSpec.ROW:
                return ("vector", ext_col(o))
            return ("scalar", ext_scalar(o, mode))

        for i, op in enumerate(self.ops):
            if isinstance(op, ReductionOp):
                kind, src = ref(op.input, BroadcastSpec.NONE, True)
                Rn = reduction_combiner(op.op)
                acc = f"r{i}"
                L.append(f"  float {acc} = {Rn}::id();")
                for p in range(P):
                    for l in range(W):
                        L.append(f"  if (col{p} + {l}u < {K}u) {acc} = {Rn}::op({acc}, {src}[{p}][{l}]);")
                L.append(f"  {acc} = mt_block_allreduce<{Rn}, {NT}>({acc}, red_scratch);")
                kinds[op.out.name] = "scalar"
                vals[op.out.name] = acc
                continue
            assert isinstance(op, ElementwiseOp)
            modes = (BroadcastSpec.NONE, op.y_broadcast, op.cond_broadcast)
            refs = [ref(o, modes[k], _is_vector_tensor(op.out)) for k, o in enumerate(op.operands)]
            tpl = elementwise_expression(op.op)
            if _is_vector_tensor(op.out):
                var = f"v{i}"
                L.append(f"  float {var}[{P}][{W}];")
                subs = {}
                for k, key in enumerate(("x", "y", "cond")[: len(refs)]):
                    kd, e = refs[k]
                    subs[key] = f"({e}[p][l])" if kd == "vector" else f"({e})"
                expr = wrap_bool(op.op, substitute(tpl, **subs))
                L.append(f"#pragma unroll\n  for (int p = 0; p < {P}; ++p) {{\n#pragma unroll\n"
                         f"    for (int l = 0; l < {W}; ++l) {var}[p][l] = {expr};\n  }}")
                kinds[op.out.name] = "vector"
            else:
                var = f"s{i}"
                subs = {}
                for k, key in enumerate(("x", "y", "cond")[: len(refs)]):
                    subs[key] = f"({refs[k][1]})"
                L.append(f"  const float {var} = {wrap_bool(op.op, substitute(tpl, **subs))};")
                kinds[op.out.name] = "scalar"
            vals[op.out.name] = var
        body = L
        L = head + LD + body
        # stores
        for op in self.ops:
            if op.out.name not in self.outputs:
                continue
            ptr = pname(op.out.buffer_key)
            v = vals[op.out.name]
            if kinds[op.out.name] == "scalar":
                L.append(f"  if (threadIdx.x == 0) {ptr}[row] = {v};")
                continue
            for p in range(P):
                if W == 4:
                    L.append(f"  if (ok{p}) mt_st_stream4({ptr} + (size_t)row * {K}ull + col{p}, "
                             f"make_float4({v}[{p}][0], {v}[{p}][1], {v}[{p}][2], {v}[{p}][3]));")
                else:
                    L.append(f"  if (ok{p}) mt_st_stream({ptr} + (size_t)row * {K}ull + col{p}, {v}[{p}][0]);")
        L.append("}")
        return "\n".join(L)


def plan_row_threads(K: int) -> tuple[int, int, int]:
    """(threads, width, chunks per thread) for a row of K columns."""
    width = 4 if K % 4 == 0 else 1
    per_row = (K + width - 1) // width
    nt = 32
    while nt < 1024 and (per_row + nt - 1) // nt > 4:
        nt *= 2
    nt = max(64, min(nt, 1024))
    chunks = (per_row + nt - 1) // nt
    return nt, width, chunks


def assemble_row_resident(decision: DecisionView, function_name: str | None) -> KernelGroup:
    ops = decision.ops
    why = row_program_check(ops)
    if why is not None:
        raise ValueError(f"row-resident vertex is not row local: {why}")
    first_vec = next(op for op in ops if isinstance(op, ReductionOp) or _is_vector_tensor(op.out))
    vec_t = first_vec.input if isinstance(first_vec, ReductionOp) else first_vec.out
    B, Mb = _rows_of(vec_t)
    K = vec_t.matrix_shape[1]
    R = B * Mb
    nt, width, chunks = plan_row_threads(K)
    outputs = tuple(decision.outputs)
    produced = {op.out.name for op in ops}
    # inputs in first-use order, then outputs
    in_keys: list[str] = []
    for op in ops:
        for t in op.inputs:
            owner = t.name if t.name in produced else (t.buffer_key if t.buffer_key in produced else None)
            if owner is None and t.buffer_key not in in_keys:
                in_keys.append(t.buffer_key)
    out_keys = [op.out.buffer_key for op in ops if op.out.name in outputs]
    bindings = (*in_keys, *out_keys)
    params = tuple(param_decl(k, writable=k in out_keys) for k in bindings)
    frag = RowResidentFragment(ops=ops, outputs=outputs, rows=R, rows_per_batch=Mb, cols=K, width=width,
                               chunks=chunks)
    # One wave: the grid is exactly the CTAs that are resident at once (threads per
    # SM 2048, registers capped at ~40 per thread by the launch bounds), each looping
    # over rows; a grid of 2048 / nt CTAs per SM would leave a partial second wave.
    blocks_per_sm = max(1, min(2048 // nt, 65536 // (nt * 40)))
    grid = max(1, min(R, SM_COUNT * blocks_per_sm))
    fn = function_name or f"row_{ops[-1].out.name}_fused"
    ctx = CodegenContext(function_name=fn, buffers=params, dims=("R", "K"), tg_x=nt, tg_y=1,
                         threadgroup_decls=("smem float red_scratch[33];",), min_blocks_per_sm=blocks_per_sm)
    return KernelGroup(kernel=Kernel(fragments=(frag,), ctx=ctx), bindings=bindings, dims=(R, K),
                       grid=(grid, 1, 1), threads=(nt, 1, 1), ops=ops, strategy=decision.strategy)
