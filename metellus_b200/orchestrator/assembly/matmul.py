"""Matmul strategies (standalone, prologue, register epilogue, shared-tile epilogue)
on the SIMT FFMA pipe — reference template: assembly/matmul.py:33-285.

Same wiring: effective device sources come from the outermost prologue primary;
input slots are deduplicated by storage key, the final output takes the next slot and
chain extras follow (so ``bindings`` match the reference's order); an aligned shape
without a shared-tile epilogue stores accumulators straight to global.
"""

from __future__ import annotations

from metellus_b200.compute.fragments import BarrierFragment, CodegenContext
from metellus_b200.compute.matmul import (
    MatmulAccumToDevFragment,
    MatmulAccumToTgFragment,
    MatmulComputeFragment,
    MatmulConfig,
    MatmulMainloopFragment,
    MatmulRegisterEpilogueFragment,
    MatmulSetupFragment,
    MatmulTgToDevFragment,
    MatmulTileMappingFragment,
    ThreadIndexFragment,
    grid_for,
    is_aligned_shape,
    select_tile_config,
)
from metellus_b200.compute.tiled_chain import TiledElementwiseChainFragment
from metellus_b200.memory.memory import TgLoadFragment
from metellus_b200.orchestrator.assembly.decision import DecisionView
from metellus_b200.orchestrator.assembly.expressions import chain_value_transform
from metellus_b200.orchestrator.assembly.extras import Extras, param_decl, pname
from metellus_b200.orchestrator.ir import MatmulOp, Tensor
from metellus_b200.orchestrator.kernel_group import FusionStrategy, KernelGroup
from metellus_b200.runtime.program import Kernel


def batch_stride_of(t: Tensor) -> int:
    return t.batch_stride if len(t.shape) == 3 else 0


def assemble_matmul(decision: DecisionView, function_name: str | None) -> KernelGroup:
    from metellus_b200.orchestrator.assembly.tc_matmul import try_assemble_tc_matmul

    tc = try_assemble_tc_matmul(decision, function_name)
    if tc is not None:
        return tc
    return assemble_matmul_simt(decision, function_name)


def assemble_matmul_simt(decision: DecisionView, function_name: str | None) -> KernelGroup:
    anchor = decision.anchor
    assert isinstance(anchor, MatmulOp)
    src_a = decision.prologue_a[0].operands[0] if decision.prologue_a else anchor.a
    src_b = decision.prologue_b[0].operands[0] if decision.prologue_b else anchor.b
    assert isinstance(src_a, Tensor) and isinstance(src_b, Tensor)
    M, K = anchor.a.matrix_shape
    N = anchor.b.matrix_shape[1]
    batch = anchor.out.batch

    tile = select_tile_config(M, K, N)
    aligned = is_aligned_shape(M, K, N, tile)
    use_register = decision.strategy is FusionStrategy.MATMUL_EPILOGUE_REGISTER
    use_tg_epilogue = bool(decision.epilogue) and not use_register
    final_out = decision.epilogue[-1].out if decision.epilogue else anchor.out
    out_key = final_out.buffer_key

    in_slots: dict[str, int] = {}
    in_bs: dict[str, int] = {}
    for t in (src_a, src_b):
        if t.buffer_key not in in_slots:
            in_slots[t.buffer_key] = len(in_slots)
            in_bs[t.buffer_key] = batch_stride_of(t)
    out_slot = len(in_slots)
    base_slots = out_slot + 1
    extras = Extras(base_slots_by_key={**in_slots, out_key: out_slot})

    a_tf = chain_value_transform(decision.prologue_a, row_var="global_row", col_var="global_col",
                                 extras=extras, base_slot=base_slots) if decision.prologue_a else None
    b_tf = chain_value_transform(decision.prologue_b, row_var="global_row", col_var="global_col",
                                 extras=extras, base_slot=base_slots) if decision.prologue_b else None
    if use_tg_epilogue:
        # Register chain secondaries read straight from global in the epilogue.
        chain_value_transform(decision.epilogue, row_var="global_row", col_var="global_col",
                              extras=extras, base_slot=base_slots)

    config = MatmulConfig(
        tile=tile, aligned=aligned and not use_tg_epilogue, M_dim_var="M", K_dim_var="K", N_dim_var="N",
        a_buffer_name=pname(src_a.buffer_key), b_buffer_name=pname(src_b.buffer_key),
        c_buffer_name=pname(out_key), a_tile_name="A_tile", b_tile_name="B_tile", c_tile_name="C_tile",
    )
    reg_epi = ()
    if use_register:
        rt = chain_value_transform(decision.epilogue, row_var="0", col_var="0", extras=extras,
                                   base_slot=base_slots)
        reg_epi = (MatmulRegisterEpilogueFragment(config=config, value_transform=rt),)

    lim = (None, None, None) if aligned else ("M", "K", "N")
    a_load = TgLoadFragment(
        name="load_A_tile", src_name=pname(src_a.buffer_key), src_row_stride=str(src_a.row_stride),
        src_col_stride=str(src_a.col_stride), row_start=f"tg.y * {tile.tile_M}u", col_start="k_chunk",
        dst_name="A_tile", tile_shape=(tile.tile_M, tile.tile_K), num_threads=tile.num_threads,
        row_limit=lim[0], col_limit=lim[1], value_transform=a_tf, transpose=True,
    )
    b_load = TgLoadFragment(
        name="load_B_tile", src_name=pname(src_b.buffer_key), src_row_stride=str(src_b.row_stride),
        src_col_stride=str(src_b.col_stride), row_start="k_chunk", col_start=f"tg.x * {tile.tile_N}u",
        dst_name="B_tile", tile_shape=(tile.tile_K, tile.tile_N), num_threads=tile.num_threads,
        row_limit=lim[1], col_limit=lim[2], value_transform=b_tf,
    )
    mainloop = MatmulMainloopFragment(
        tile_K=tile.tile_K,
        fragments=(a_load, b_load, BarrierFragment("inputs_ready"), MatmulComputeFragment(config),
                   BarrierFragment("compute_done")),
        K_dim_var="K",
    )
    if use_tg_epilogue:
        store = [
            MatmulAccumToTgFragment(config), BarrierFragment("c_tile_ready"),
            TiledElementwiseChainFragment(
                chain=decision.epilogue, primary_tile="C_tile", tile_shape=(tile.tile_M, tile.tile_N),
                num_threads=tile.num_threads, y_tile_for={}, row_origin=f"tg.y * {tile.tile_M}u",
                col_origin=f"tg.x * {tile.tile_N}u", row_limit="M", col_limit="N",
            ),
            BarrierFragment("epilogue_done"), MatmulTgToDevFragment(config),
        ]
    elif config.aligned:
        store = [*reg_epi, MatmulAccumToDevFragment(config)]
    else:
        store = [*reg_epi, MatmulAccumToTgFragment(config), BarrierFragment("c_tile_ready"),
                 MatmulTgToDevFragment(config)]
    fragments = (MatmulTileMappingFragment(), ThreadIndexFragment(tile), MatmulSetupFragment(config),
                 mainloop, *store)
    decls = [
        f"smem float A_tile[{tile.tile_K}][{tile.tile_M + tile.a_pad}];",
        f"smem float B_tile[{tile.tile_K}][{tile.tile_N + tile.b_pad}];",
    ]
    if not config.aligned:
        decls.append(f"smem float C_tile[{tile.tile_M}][{tile.tile_N + tile.c_pad}];")
    bindings = (*in_slots.keys(), out_key, *extras.bindings)
    params = tuple(param_decl(k, writable=(k == out_key)) for k in bindings)
    bstrides = tuple([in_bs[k] for k in in_slots] + [batch_stride_of(final_out)] + extras.batch_strides)
    fn = function_name or f"matmul_{anchor.out.name}_fused"
    ctx = CodegenContext(function_name=fn, buffers=params, dims=("M", "K", "N"), tg_x=tile.tg_x,
                         tg_y=tile.tg_y, threadgroup_decls=tuple(decls),
                         batch_strides=bstrides if batch > 1 else ())
    gx, gy, _ = grid_for(M, N, tile)
    return KernelGroup(
        kernel=Kernel(fragments=fragments, ctx=ctx), bindings=bindings, dims=(M, K, N),
        grid=(gx, gy, batch), threads=(tile.tg_x, tile.tg_y, 1), ops=decision.ops,
        strategy=decision.strategy, pipe="ffma",
    )
