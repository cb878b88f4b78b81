"""FUSED_ATTENTION strategy (B200): ``O = softmax(f(Q @ K^T)) @ V`` in one kernel.

The reference lowers the primitive attention program to five kernels per head
(QK^T with a register epilogue, max-reduce, [sub, exp], sum-reduce, divide prologue +
PV), materialising the S x S scores and probabilities in memory several times. This
pass recognises the subgraph

    s  = matmul(Q, Kt)                    (Kt a transposed view, K stored row major)
    s' = f(s)                             (lane-agnostic scalar chain, e.g. * 0.125)
    mx = max(s', axis=-1);   sub = s' - view(mx) (col);   e = exp(sub)
    sm = sum(e, axis=-1);    p = e / view(sm) (col);      O = matmul(p, V)

and fuses it into one flash-style kernel (online softmax over key blocks); the row
statistics ``mx`` and ``sm`` are still written when the program exposes them. Only the
S x S intermediates disappear.

Head dim 64 with whole 64-key blocks runs on the tensor cores (tcgen05, 3xTF32,
``mt_attn_tc.cuh``: TMA-fed K / V blocks, Q and P in tensor memory); other shapes run
the FFMA kernel (``mt_attn.cuh``).
"""

from __future__ import annotations

from dataclasses import dataclass

from metellus_b200.compute.device_lib import header
from metellus_b200.compute.elementwise import BroadcastSpec
from metellus_b200.compute.fragments import CodegenContext, TgmemAccess
from metellus_b200.orchestrator.assembly.decision import DecisionView, is_lane_agnostic_pred
from metellus_b200.orchestrator.assembly.expressions import build_reduction_epilogue_transform
from metellus_b200.orchestrator.assembly.extras import param_decl, pname
from metellus_b200.orchestrator.graph import Graph
from metellus_b200.orchestrator.ir import ElementwiseOp, MatmulOp, ReductionOp, Tensor
from metellus_b200.orchestrator.kernel_group import KernelGroup
from metellus_b200.orchestrator.kernel_group import STATUS_BYTES, STATUS_KEY
from metellus_b200.runtime.program import Kernel, TmapSpec


@dataclass(frozen=True)
class AttentionMatch:
    qk: MatmulOp
    score_chain: tuple[ElementwiseOp, ...]
    mx: ReductionOp
    sub: ElementwiseOp
    ex: ElementwiseOp
    sm: ReductionOp
    div: ElementwiseOp
    pv: MatmulOp

    @property
    def ops(self):
        return (self.qk, *self.score_chain, self.mx, self.sub, self.ex, self.sm, self.div, self.pv)


def _owner(t: Tensor) -> str:
    return t.buffer_key


def find_attention(ops) -> AttentionMatch | None:
    """Match the attention pattern starting from any matmul in ``ops`` (a program or
    the union of vertex ops)."""
    by_out = {op.out.name: op for op in ops}
    readers: dict[str, list] = {}
    for op in ops:
        for t in op.inputs:
            readers.setdefault(t.name, []).append(op)
            if t.buffer_key != t.name:
                readers.setdefault(t.buffer_key, []).append(op)

    def only_reader(name):
        r = readers.get(name, [])
        return r[0] if len(r) == 1 else None

    for qk in ops:
        if not isinstance(qk, MatmulOp):
            continue
        chain = []
        cur = qk.out.name
        nxt = only_reader(cur)
        while isinstance(nxt, ElementwiseOp) and is_lane_agnostic_pred(nxt) and nxt.operands[0].name == cur:
            chain.append(nxt)
            cur = nxt.out.name
            nxt = only_reader(cur)
        rs = readers.get(cur, [])
        mx = next((o for o in rs if isinstance(o, ReductionOp) and o.op == "max"), None)
        sub = next((o for o in rs if isinstance(o, ElementwiseOp) and o.op == "subtract"), None)
        if mx is None or sub is None or len(rs) != 2:
            continue
        if not (sub.operands[0].name == cur and sub.y_broadcast is BroadcastSpec.COL
                and isinstance(sub.operands[1], Tensor) and _owner(sub.operands[1]) == mx.out.name):
            continue
        ex = only_reader(sub.out.name)
        if not (isinstance(ex, ElementwiseOp) and ex.op == "exp"):
            continue
        rs = readers.get(ex.out.name, [])
        sm = next((o for o in rs if isinstance(o, ReductionOp) and o.op == "sum"), None)
        div = next((o for o in rs if isinstance(o, ElementwiseOp) and o.op == "div"), None)
        if sm is None or div is None or len(rs) != 2:
            continue
        if not (div.operands[0].name == ex.out.name and div.y_broadcast is BroadcastSpec.COL
                and isinstance(div.operands[1], Tensor) and _owner(div.operands[1]) == sm.out.name):
            continue
        pv = only_reader(div.out.name)
        if not (isinstance(pv, MatmulOp) and pv.a.name == div.out.name):
            continue
        # the row stats may only be read through the two col-broadcast views
        if any(o not in (sub,) for o in readers.get(mx.out.name, [])) or \
                any(o not in (div,) for o in readers.get(sm.out.name, [])):
            continue
        return AttentionMatch(qk, tuple(chain), mx, sub, ex, sm, div, pv)
    return None


def attention_supported(m: AttentionMatch) -> bool:
    Q, Kt, V = m.qk.a, m.qk.b, m.pv.b
    D = Q.shape[-1]
    return (D % 64 == 0 and D <= 128 and Q.col_stride == 1 and Kt.row_stride == 1 and V.col_stride == 1
            and V.shape[-1] == D and len(Q.shape) == len(Kt.shape) == len(V.shape))


def match_attention(graph: Graph, blacklist):
    """Fusion pass: collapse the vertices holding one attention subgraph."""
    all_ops = [op for v in graph.vertices for op in v.ops]
    m = find_attention(all_ops)
    if m is None or not attention_supported(m):
        return None
    ids = {id(o) for o in m.ops}
    members = [v for v in graph.vertices if any(id(o) in ids for o in v.ops)]
    if any(id(o) not in ids for v in members for o in v.ops):
        return None
    if len(members) == 1:
        return None  # already fused
    sig = frozenset(id(o) for v in members for o in v.ops)
    if sig in blacklist:
        return None
    ops = tuple(op for _, op in sorted(((graph.op_index[id(o)], o) for v in members for o in v.ops),
                                       key=lambda p: p[0]))
    try:
        g = graph.replace(absorbed=tuple(members), ops=ops)
    except ValueError:
        return None
    merged = next(v for v in g.vertices if id(v) not in {id(x) for x in graph.vertices})
    internal = {m.qk.out.name, *(o.out.name for o in m.score_chain), m.sub.out.name, m.ex.out.name,
                m.div.out.name}
    if internal & set(merged.outputs):
        return None  # an S x S intermediate is needed elsewhere: keep the unfused plan
    return g


@dataclass(frozen=True)
class AttentionFragment:
    d: int
    score_expr: str
    q: str
    k: str
    v: str
    o: str
    mx: str
    sm: str
    sq: int
    sk: int
    q_rs: int
    k_rs: int
    v_rs: int
    o_rs: int
    name: str = "attention"
    kind: str = "compute"

    @property
    def tgmem_accesses(self) -> tuple[TgmemAccess, ...]:
        n = _smem_floats(self.d)
        return (TgmemAccess("attn_arena", "readwrite", n, (1, n)),)

    def render(self, ctx: CodegenContext) -> str:
        return (
            f"auto score = [=](float x) -> float {{ return {self.score_expr}; }};\n"
            f"mt_attn_fwd_simt<{self.d}>({self.q}, {self.k}, {self.v}, {self.o}, {self.mx}, {self.sm}, "
            f"{self.sq}, {self.sk}, {self.q_rs}ll, {self.k_rs}ll, {self.v_rs}ll, {self.o_rs}ll, score, attn_arena);"
        )


def _smem_floats(d: int) -> int:
    bq = bk = 64
    return d * (bq + 4) + d * (bk + 4) + bk * (d + 4) + bk * (bq + 4)


@dataclass(frozen=True)
class TcAttentionFragment:
    score_expr: str
    o: str
    mx: str
    sm: str
    sq: int
    sk: int
    o_rs: int
    name: str = "attention_tc"
    kind: str = "compute"

    @property
    def tgmem_accesses(self) -> tuple[TgmemAccess, ...]:
        return (TgmemAccess("attn_arena", "readwrite", TC_ARENA_FLOATS, (1, TC_ARENA_FLOATS)),)

    def render(self, ctx: CodegenContext) -> str:
        return (
            f"auto score = [=](float x) -> float {{ return {self.score_expr}; }};\n"
            f"mt_attn_fwd_tc(&tm_q, &tm_k, &tm_v, {self.o}, {self.mx}, {self.sm}, {self.sq}, {self.sk}, "
            f"{self.o_rs}ll, score, g_status, attn_arena);"
        )


# mt_fa_layout::kBytes (Q / Q lo 32 KB + two 64 KB K/V stages + half-row exchange +
# barriers) plus 1 KB for aligning the arena to the 128-byte swizzle atom.
TC_ARENA_FLOATS = (32768 + 2 * 65536 + 2048 + 32 * 8 + 16 + 1024) // 4


def _tc_attention_ok(Q: Tensor, Kt: Tensor, V: Tensor, O: Tensor, D: int, Sk: int) -> bool:
    from metellus_b200.orchestrator.assembly.tc_matmul import _fits_cap, tc_enabled

    def bs(t: Tensor) -> int:
        return t.batch_stride if len(t.shape) == 3 else 0

    aligned = all(x * 4 % 16 == 0 for x in (Q.row_stride, Kt.col_stride, V.row_stride, bs(Q), bs(Kt), bs(V)))
    return (tc_enabled() and D == 64 and Sk % 64 == 0 and aligned and O.col_stride == 1
            and O.row_stride % 4 == 0 and _fits_cap(TC_ARENA_FLOATS * 4))


def assemble_attention(decision: DecisionView, function_name: str | None) -> KernelGroup:
    m = find_attention(decision.ops)
    if m is None:
        raise ValueError("fused-attention vertex does not hold the attention pattern")
    Q, Kt, V, O = m.qk.a, m.qk.b, m.pv.b, m.pv.out
    batched = len(Q.shape) == 3
    B = Q.shape[0] if batched else 1
    Sq, D = Q.shape[-2], Q.shape[-1]
    Sk = Kt.shape[-1]
    outputs = set(decision.outputs)
    in_keys = []
    for t in (Q, Kt, V):
        if t.buffer_key not in in_keys:
            in_keys.append(t.buffer_key)
    out_keys = [O.buffer_key]
    stat_mx = m.mx.out.buffer_key if m.mx.out.name in outputs else None
    stat_sm = m.sm.out.buffer_key if m.sm.out.name in outputs else None
    out_keys += [k for k in (stat_mx, stat_sm) if k is not None]
    bindings = (*in_keys, *out_keys)
    params = tuple(param_decl(k, writable=k in out_keys) for k in bindings)

    def bs(t: Tensor) -> int:
        return t.batch_stride if len(t.shape) == 3 else 0

    strides = {Q.buffer_key: bs(Q), Kt.buffer_key: bs(Kt), V.buffer_key: bs(V), O.buffer_key: bs(O)}
    if stat_mx:
        strides[stat_mx] = Sq if batched else 0
    if stat_sm:
        strides[stat_sm] = Sq if batched else 0
    score = build_reduction_epilogue_transform(m.score_chain)("x")
    if _tc_attention_ok(Q, Kt, V, O, D, Sk):
        return _assemble_tc(decision, m, function_name, bindings, params, strides, batched, B, Sq, Sk, D,
                            stat_mx, stat_sm, score)
    frag = AttentionFragment(
        d=D, score_expr=score, q=pname(Q.buffer_key), k=pname(Kt.buffer_key), v=pname(V.buffer_key),
        o=pname(O.buffer_key), mx=pname(stat_mx) if stat_mx else "nullptr",
        sm=pname(stat_sm) if stat_sm else "nullptr", sq=Sq, sk=Sk, q_rs=Q.row_stride, k_rs=Kt.col_stride,
        v_rs=V.row_stride, o_rs=O.row_stride,
    )
    fn = function_name or f"attention_{O.name}_fused"
    ctx = CodegenContext(
        function_name=fn, buffers=params, dims=("B", "S", "D"), tg_x=256, tg_y=1,
        threadgroup_decls=(f"smem float attn_arena[{_smem_floats(D)}];",), helpers=(header("mt_attn.cuh"),),
        batch_strides=tuple(strides[k] for k in bindings) if batched else (),
    )
    return KernelGroup(kernel=Kernel(fragments=(frag,), ctx=ctx), bindings=bindings, dims=(B, Sq, D),
                       grid=(-(-Sq // 64), 1, B), threads=(256, 1, 1), ops=decision.ops,
                       strategy=decision.strategy, pipe="ffma")


def _assemble_tc(decision, m, function_name, bindings, params, strides, batched, B, Sq, Sk, D, stat_mx, stat_sm,
                 score) -> KernelGroup:
    Q, Kt, V, O = m.qk.a, m.qk.b, m.pv.b, m.pv.out

    def bs(t: Tensor, rows: int, rs: int) -> int:
        return t.batch_stride if len(t.shape) == 3 else rows * rs

    qi, ki, vi = bindings.index(Q.buffer_key), bindings.index(Kt.buffer_key), bindings.index(V.buffer_key)
    # Q, K: K-major 128-byte-swizzled boxes of 32 d x rows; V: d-contiguous (MN-major for
    # the P V product) boxes {32 d, 32 keys, 2 d-chunks} on 32-byte swizzle atoms.
    tmaps = (
        TmapSpec(qi, (D, Sq, B), (Q.row_stride * 4, bs(Q, Sq, Q.row_stride) * 4), (32, 128, 1)),
        TmapSpec(ki, (D, Sk, B), (Kt.col_stride * 4, bs(Kt, Sk, Kt.col_stride) * 4), (32, 64, 1)),
        TmapSpec(vi, (32, Sk, D // 32, B), (V.row_stride * 4, 128, bs(V, Sk, V.row_stride) * 4), (32, 32, 2, 1),
                 swizzle=4),
    )
    frag = TcAttentionFragment(
        score_expr=score, o=pname(O.buffer_key), mx=pname(stat_mx) if stat_mx else "nullptr",
        sm=pname(stat_sm) if stat_sm else "nullptr", sq=Sq, sk=Sk, o_rs=O.row_stride,
    )
    fn = function_name or f"attention_{O.name}_fused"
    ctx = CodegenContext(
        function_name=fn, buffers=params + ("int* g_status",), dims=("B", "S", "D"), tg_x=512, tg_y=1,
        threadgroup_decls=(f"smem float attn_arena[{TC_ARENA_FLOATS}];",),
        helpers=(header("mt_tc.cuh"), header("mt_attn_tc.cuh")),
        extra_params=("const __grid_constant__ mt_tmap tm_q", "const __grid_constant__ mt_tmap tm_k",
                      "const __grid_constant__ mt_tmap tm_v"),
        batch_strides=tuple(strides[k] for k in bindings) if batched else (),
        min_blocks_per_sm=1,
    )
    return KernelGroup(kernel=Kernel(fragments=(frag,), ctx=ctx), bindings=bindings, dims=(B, Sq, D),
                       grid=(-(-Sq // 128), 1, B), threads=(512, 1, 1), ops=decision.ops,
                       strategy=decision.strategy, pipe="tcgen05", tmaps=tmaps,
                       scratch=((STATUS_KEY, STATUS_BYTES),))
