"""The bounded-wait path of the tcgen05 GEMM, exercised on purpose without a fault.

Every mbarrier wait in the tensor-core kernels is bounded by wall time; on timeout the
waiting thread writes a code into the kernel's status word, the CTA's roles leave
their loops, in-flight copies are drained, tensor memory is freed and the kernel
returns normally, and the host raises when it reads the status. This test builds one
small GEMM with the wait limit shortened to 1 ms and the TMA producer told to stop
after two k-tiles (``MT_TEST_STALL_KTILE``), so a consumer's wait runs out: a barrier
that nothing will complete, not a fault. It checks that the host raises, and that the
next normal launch on the same GPU (same context) computes the right answer. The
reference raises only on Metal errors (metal_backend.mm:230-232)."""

from __future__ import annotations

import numpy as np
import pytest

from metellus_b200 import run
from metellus_b200.api.run import compile_program
from metellus_b200.orchestrator.scheduler import schedule
from oracle.ir_eval import evaluate
from tests.test_gpu_matmul import _mm
from tests.tolerances import assert_matmul_close

pytestmark = pytest.mark.gpu

STALL = "#define MT_WAIT_LIMIT_NS 1000000ull\n#define MT_TEST_STALL_KTILE 2\n"


def test_wait_timeout_reports_and_context_survives(cuda_device):
    ops, out = _mm(256, 256, 256, seed=5)
    groups = compile_program(ops)
    g = groups[0]
    # the one-CTA kernel (no cluster): 8 k-tiles, the producer stops before the third
    assert len(groups) == 1 and g.pipe == "tcgen05" and g.cluster_x == 1, (g.pipe, g.cluster_x)
    g.kernel._source = STALL + g.kernel.source
    with pytest.raises(RuntimeError, match="timed out"):
        schedule(ops, groups).run()
    res = run(ops)
    r64, r32 = evaluate(ops, np.float64), evaluate(ops, np.float32)
    assert_matmul_close(res.env[out], r64[out], r32[out], what="after a timed-out launch")
