"""``KernelGroup``: one fused CUDA kernel plus everything needed to launch it.

The 12 reference strategies (kernel_group.py:23-56) keep their names and meaning.
B200-only strategies are appended; they are produced only by the B200 fusion passes
(``orchestrator.fusion.B200_PASSES``):

* ``ELEMENTWISE_DAG``   — several elementwise chains over one element space fused into
  one streaming kernel (multi-root loads, possibly several materialised outputs).
* ``ROW_RESIDENT``      — reductions plus the elementwise ops around them, all over one
  row space, with each row held in registers for the whole program (softmax,
  layernorm): one HBM read and one write per element.
* ``FUSED_ATTENTION``   — matmul -> scale -> row softmax -> matmul, flash style.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from enum import StrEnum

from metellus_b200.orchestrator.ir import Op
from metellus_b200.runtime.program import Kernel


STATUS_KEY = "__mt_status"
STATUS_BYTES = 64


class FusionStrategy(StrEnum):
    STANDALONE_MATMUL = "standalone_matmul"
    STANDALONE_ELEMENTWISE = "standalone_elementwise"
    STANDALONE_REDUCTION = "standalone_reduction"
    MATMUL_EPILOGUE_REGISTER = "matmul_epilogue_register"
    MATMUL_EPILOGUE_TG = "matmul_epilogue_tg"
    ELEMENTWISE_PROLOGUE_MATMUL = "elementwise_prologue_matmul"
    ELEMENTWISE_PROLOGUE_REDUCTION = "elementwise_prologue_reduction"
    REDUCTION_EPILOGUE = "reduction_epilogue"
    ELEMENTWISE_CHAIN = "elementwise_chain"
    STANDALONE_SHAPE = "standalone_shape"
    MULTI_PRODUCER_CONVERGENT = "multi_producer_convergent"
    DIAMOND_SHARED = "diamond_shared"
    # B200-only strategies.
    ELEMENTWISE_DAG = "elementwise_dag"
    ROW_RESIDENT = "row_resident"
    FUSED_ATTENTION = "fused_attention"
    DUAL_GEMM_EPILOGUE = "dual_gemm_epilogue"


@dataclass(frozen=True)
class KernelGroup:
    """One kernel ready to dispatch (kernel_group.py:59-82).

    ``bindings`` are env keys in kernel-parameter order; ``dims`` the runtime dim
    values; ``grid``/``threads`` the CUDA launch shape (blocks, threads per block).
    ``pipe`` names the arithmetic pipe of a matmul-bearing group ("ffma" SIMT tiles
    or "tcgen05" 3xTF32 tensor-core tiles); ``tmaps`` lists the TMA tensor maps the
    backend encodes for the launch (empty for plain kernels); ``scratch`` lists
    (key, nbytes) buffers the kernel takes after its bindings — zero-initialised
    device memory owned by the runtime, e.g. the ``STATUS_KEY`` word that bounded
    waits write on timeout."""

    kernel: Kernel
    bindings: tuple[str, ...]
    dims: tuple[int, ...]
    grid: tuple[int, int, int]
    threads: tuple[int, int, int]
    ops: tuple[Op, ...]
    strategy: FusionStrategy
    pipe: str = ""
    tmaps: tuple = field(default=())
    scratch: tuple = field(default=())
    cluster_x: int = 1

    @property
    def outputs(self) -> tuple[str, ...]:
        return tuple(op.out.name for op in self.ops if op.out.name in self.bindings)
