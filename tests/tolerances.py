"""Parity tolerances used by the GPU tests (stated in one place).

* EXACT: pure add / mul / max / select chains are compared bit for bit with the fp32
  oracle (``np.array_equal``, NaNs equal).
* Transcendental / reduction programs: |gpu - fp64| <= ELEM_ABS + ELEM_REL * |fp64|
  per element, with ELEM_REL = 1e-6 (2-ulp scale) and a small absolute floor.
* Matmul-bearing programs: normwise relative error ||gpu - fp64||_F / ||fp64||_F <=
  MATMUL_NORMWISE (1e-5), and no worse than MATMUL_VS_FP32 x the fp32 oracle's own
  normwise error (the MLX-CPU fp32 stand-in).
"""

import numpy as np

ELEM_REL = 1e-6
ELEM_ABS = 2e-7
MATMUL_NORMWISE = 1e-5
MATMUL_VS_FP32 = 4.0


def normwise(a, ref) -> float:
    a = np.asarray(a, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.linalg.norm((a - ref).ravel()) / max(np.linalg.norm(ref.ravel()), 1e-300))


def assert_elementwise_close(got, ref64, rel=ELEM_REL, abs_=ELEM_ABS, what=""):
    got = np.asarray(got, dtype=np.float64)
    ref64 = np.asarray(ref64, dtype=np.float64)
    err = np.abs(got - ref64)
    bound = abs_ + rel * np.abs(ref64)
    bad = ~(err <= bound) & ~(np.isnan(got) & np.isnan(ref64))
    if bad.any():
        i = np.unravel_index(np.argmax(np.where(bad, err - bound, -np.inf)), err.shape)
        raise AssertionError(f"{what}: {int(bad.sum())} elements out of tolerance; worst at {i}: "
                             f"got {got[i]!r} ref {ref64[i]!r} err {err[i]:.3e} bound {bound[i]:.3e}")


def assert_matmul_close(got, ref64, ref32, what=""):
    e = normwise(got, ref64)
    e32 = normwise(ref32, ref64)
    assert e <= MATMUL_NORMWISE, f"{what}: normwise error {e:.3e} > {MATMUL_NORMWISE}"
    assert e <= max(MATMUL_VS_FP32 * e32, 1e-7), f"{what}: normwise error {e:.3e} vs fp32 oracle {e32:.3e}"
