"""Two matmul anchors + one merge elem on the SIMT pipe (reference template:
assembly/multi_anchor.py:50-355): per-anchor accumulators, one shared A-load per
k-chunk in the diamond case (both anchors read the same A with matching K) or two
sequential mainloops otherwise, both accumulator sets drained to shared tiles, the
merge applied on the tiles and the result stored."""

from __future__ import annotations

from metellus_b200.compute.fragments import BarrierFragment, CodegenContext
from metellus_b200.compute.matmul import (
    MatmulAccumToTgFragment,
    MatmulComputeFragment,
    MatmulConfig,
    MatmulMainloopFragment,
    MatmulSetupFragment,
    MatmulTileMappingFragment,
    ThreadIndexFragment,
    grid_for,
    select_tile_config,
)
from metellus_b200.compute.tiled_chain import TiledElementwiseChainFragment
from metellus_b200.memory.memory import TgLoadFragment, TgStoreFragment
from metellus_b200.orchestrator.assembly.decision import DecisionView
from metellus_b200.orchestrator.assembly.expressions import chain_value_transform
from metellus_b200.orchestrator.assembly.extras import Extras, param_decl, pname
from metellus_b200.orchestrator.assembly.matmul import batch_stride_of
from metellus_b200.orchestrator.ir import Tensor
from metellus_b200.orchestrator.kernel_group import KernelGroup
from metellus_b200.runtime.program import Kernel


def assemble_multi_anchor(decision: DecisionView, function_name: str | None) -> KernelGroup:
    from metellus_b200.orchestrator.assembly.tc_matmul import try_assemble_tc_multi_anchor

    tc = try_assemble_tc_multi_anchor(decision, function_name)
    if tc is not None:
        return tc
    if decision.epilogue:
        raise ValueError("dual-GEMM vertex: the tcgen05 assembly rejected it (the fusion pass "
                         "only builds one when the tensor-core path accepts the anchors)")
    a0, a1 = decision.anchors
    merge = decision.merge_elem
    assert merge is not None
    M, N = a0.out.matrix_shape
    K0, K1 = a0.a.matrix_shape[1], a1.a.matrix_shape[1]
    batch = a0.out.batch
    shared_a = decision.shared_a and K0 == K1
    pa = decision.prologues_a or ((), ())
    pb = decision.prologues_b or ((), ())
    src_a = tuple(pa[i][0].operands[0] if pa[i] else decision.anchors[i].a for i in range(2))
    src_b = tuple(pb[i][0].operands[0] if pb[i] else decision.anchors[i].b for i in range(2))
    final_out = merge.out
    out_key = final_out.buffer_key
    tile = select_tile_config(M, max(K0, K1), N)

    cands = (src_a[0], src_b[0], src_b[1]) if shared_a else (src_a[0], src_b[0], src_a[1], src_b[1])
    in_keys: list[str] = []
    in_bs: list[int] = []
    for t in cands:
        assert isinstance(t, Tensor)
        if t.buffer_key not in in_keys:
            in_keys.append(t.buffer_key)
            in_bs.append(batch_stride_of(t))
    out_slot = len(in_keys)
    base_slots = out_slot + 1
    extras = Extras(base_slots_by_key={**{k: i for i, k in enumerate(in_keys)}, out_key: out_slot})
    tf_a = tuple(chain_value_transform(pa[i], row_var="global_row", col_var="global_col", extras=extras,
                                       base_slot=base_slots) if pa[i] else None for i in range(2))
    tf_b = tuple(chain_value_transform(pb[i], row_var="global_row", col_var="global_col", extras=extras,
                                       base_slot=base_slots) if pb[i] else None for i in range(2))
    if shared_a:
        dim_names, dim_vals = ("M", "K", "N"), (M, K0, N)
    else:
        dim_names, dim_vals = ("M", "K0", "K1", "N"), (M, K0, K1, N)
    cfgs = tuple(
        MatmulConfig(tile=tile, aligned=False, M_dim_var="M", K_dim_var="K" if shared_a else f"K{i}",
                     N_dim_var="N", a_buffer_name=pname(src_a[i].buffer_key),
                     b_buffer_name=pname(src_b[i].buffer_key), c_buffer_name=pname(out_key),
                     a_tile_name="A_tile" if shared_a else f"A{i}_tile", b_tile_name=f"B{i}_tile",
                     c_tile_name=f"C{i}_tile")
        for i in range(2)
    )
    sfx = ("_0", "_1")
    setup = [MatmulTileMappingFragment(), ThreadIndexFragment(tile),
             MatmulSetupFragment(cfgs[0], accumulator_suffix=sfx[0]),
             MatmulSetupFragment(cfgs[1], accumulator_suffix=sfx[1], emit_thread_coords=False)]

    def load(i: int, side: str) -> TgLoadFragment:
        src = src_a[i] if side == "A" else src_b[i]
        tname = ("A_tile" if shared_a else f"A{i}_tile") if side == "A" else f"B{i}_tile"
        kv = cfgs[i].K_dim_var
        if side == "A":
            return TgLoadFragment(
                name=f"load_{tname}", src_name=pname(src.buffer_key), src_row_stride=str(src.row_stride),
                src_col_stride=str(src.col_stride), row_start=f"tg.y * {tile.tile_M}u", col_start="k_chunk",
                dst_name=tname, tile_shape=(tile.tile_M, tile.tile_K), num_threads=tile.num_threads,
                row_limit="M", col_limit=kv, value_transform=tf_a[i], transpose=True)
        return TgLoadFragment(
            name=f"load_{tname}", src_name=pname(src.buffer_key), src_row_stride=str(src.row_stride),
            src_col_stride=str(src.col_stride), row_start="k_chunk", col_start=f"tg.x * {tile.tile_N}u",
            dst_name=tname, tile_shape=(tile.tile_K, tile.tile_N), num_threads=tile.num_threads,
            row_limit=kv, col_limit="N", value_transform=tf_b[i])

    if shared_a:
        loops = [MatmulMainloopFragment(
            tile_K=tile.tile_K,
            fragments=(load(0, "A"), load(0, "B"), load(1, "B"), BarrierFragment("inputs_ready"),
                       MatmulComputeFragment(cfgs[0], accumulator_suffix=sfx[0]),
                       MatmulComputeFragment(cfgs[1], accumulator_suffix=sfx[1]),
                       BarrierFragment("compute_done")),
            K_dim_var="K")]
    else:
        loops = [MatmulMainloopFragment(
            tile_K=tile.tile_K,
            fragments=(load(i, "A"), load(i, "B"), BarrierFragment(f"inputs{i}_ready"),
                       MatmulComputeFragment(cfgs[i], accumulator_suffix=sfx[i]),
                       BarrierFragment(f"compute{i}_done")),
            K_dim_var=cfgs[i].K_dim_var) for i in range(2)]
    # merge secondary operands other than the second anchor come from global.
    other = [o for o in merge.operands[1:] if isinstance(o, Tensor) and o.name != a1.out.name
             and o.name != a0.out.name]
    for o in other:
        extras.add_tensor(o, base_slots)
    y_tile = {0: "C1_tile"} if (isinstance(merge.operands[1], Tensor)
                                and merge.operands[1].name == a1.out.name) else {}
    if isinstance(merge.operands[0], Tensor) and merge.operands[0].name == a1.out.name:
        primary_tile, y_tile = "C1_tile", {0: "C0_tile"}
    else:
        primary_tile = "C0_tile"
    merge_frag = TiledElementwiseChainFragment(
        chain=(merge,), primary_tile=primary_tile, tile_shape=(tile.tile_M, tile.tile_N),
        num_threads=tile.num_threads, y_tile_for=y_tile, row_origin=f"tg.y * {tile.tile_M}u",
        col_origin=f"tg.x * {tile.tile_N}u", row_limit="M", col_limit="N")
    store = TgStoreFragment(
        name="store_merged", src_name=primary_tile, dst_name=pname(out_key), dst_row_stride="N",
        row_start=f"tg.y * {tile.tile_M}u", col_start=f"tg.x * {tile.tile_N}u",
        tile_shape=(tile.tile_M, tile.tile_N), num_threads=tile.num_threads, row_limit="M", col_limit="N")
    fragments = (*setup, *loops,
                 MatmulAccumToTgFragment(cfgs[0], accumulator_suffix=sfx[0]),
                 MatmulAccumToTgFragment(cfgs[1], accumulator_suffix=sfx[1], emit_tg_coords=False),
                 BarrierFragment("c_tiles_ready"), merge_frag, BarrierFragment("merge_done"), store)
    decls = []
    if shared_a:
        decls.append(f"smem float A_tile[{tile.tile_K}][{tile.tile_M + tile.a_pad}];")
    else:
        decls += [f"smem float A{i}_tile[{tile.tile_K}][{tile.tile_M + tile.a_pad}];" for i in range(2)]
    decls += [f"smem float B{i}_tile[{tile.tile_K}][{tile.tile_N + tile.b_pad}];" for i in range(2)]
    decls += [f"smem float C{i}_tile[{tile.tile_M}][{tile.tile_N + tile.c_pad}];" for i in range(2)]
    bindings = (*in_keys, out_key, *extras.bindings)
    params = tuple(param_decl(k, writable=(k == out_key)) for k in bindings)
    bstrides = tuple(in_bs + [batch_stride_of(final_out)] + extras.batch_strides)
    fn = function_name or f"multi_anchor_{final_out.name}_fused"
    ctx = CodegenContext(function_name=fn, buffers=params, dims=dim_names, tg_x=tile.tg_x, tg_y=tile.tg_y,
                         threadgroup_decls=tuple(decls), batch_strides=bstrides if batch > 1 else ())
    gx, gy, _ = grid_for(M, N, tile)
    return KernelGroup(kernel=Kernel(fragments=fragments, ctx=ctx), bindings=bindings, dims=dim_vals,
                       grid=(gx, gy, batch), threads=(tile.tg_x, tile.tg_y, 1), ops=decision.ops,
                       strategy=decision.strategy, pipe="ffma")
