"""GPU parity of matmul groups on both pipes (tcgen05 3xTF32 and SIMT FFMA) against
the fp64 oracle: normwise relative error <= 1e-5 and no worse than 4x the fp32 oracle
(tests/tolerances.py). Covers aligned and ragged M / N / K, a transposed-view B
(K^T, K-major B tiles), an A-side prologue, shared-tile epilogues and the diamond."""

from __future__ import annotations

import numpy as np
import pytest

from metellus_b200 import Operations, run
from oracle.ir_eval import evaluate
from tests.tolerances import assert_matmul_close

pytestmark = pytest.mark.gpu


def _mm(M, K, N, *, bias=False, relu=False, transpose_b=False, prologue=False, seed=0):
    r = np.random.default_rng(seed)
    A = r.normal(0, 1, (M, K)).astype(np.float32)
    ops = Operations()
    ops.from_numpy(A, "A")
    if transpose_b:
        Bt = r.normal(0, 1, (N, K)).astype(np.float32)
        ops.from_numpy(Bt, "Bt")
        ops.transpose("Bt", out="B")
    else:
        ops.from_numpy(r.normal(0, 1, (K, N)).astype(np.float32), "B")
    a = "A"
    if prologue:
        ops.elementwise("max", out="Ar", operands=("A", -0.5))
        a = "Ar"
    ops.matmul(a=a, b="B", out="C")
    last = "C"
    if bias:
        ops.from_numpy(r.normal(0, 1, (1, N)).astype(np.float32), "bias")
        ops.elementwise("add", out="Cb", operands=("C", "bias"), y_broadcast="row")
        last = "Cb"
    if relu:
        ops.elementwise("max", out="Y", operands=(last, 0.0))
        last = "Y"
    return ops, last


CASES = [
    dict(M=256, K=256, N=256),
    dict(M=1024, K=1024, N=1024, bias=True, relu=True),
    dict(M=200, K=100, N=96),            # ragged M and K
    dict(M=128, K=64, N=100, transpose_b=True),   # K-major B, N not a multiple of 32
    dict(M=384, K=512, N=256, transpose_b=True, bias=True),
    dict(M=256, K=96, N=160, prologue=True, relu=True),
]


@pytest.mark.parametrize("pipe", ["tcgen05", "ffma"])
@pytest.mark.parametrize("case", CASES, ids=lambda c: "x".join(str(c[k]) for k in "MKN") + "".join(
    k[0] for k, v in c.items() if v is True))
def test_matmul_pipes(cuda_device, monkeypatch, pipe, case):
    monkeypatch.setenv("METELLUS_TC", "1" if pipe == "tcgen05" else "0")
    ops, out = _mm(**case)
    res = run(ops)
    assert len(res.groups) == 1
    if pipe == "tcgen05":
        assert res.groups[0].pipe == "tcgen05", res.groups[0].pipe
    r64 = evaluate(ops, np.float64)
    r32 = evaluate(ops, np.float32)
    assert_matmul_close(res.env[out], r64[out], r32[out], what=f"{pipe} {case}")


@pytest.mark.parametrize("pipe", ["tcgen05", "ffma"])
def test_diamond_shared_a(cuda_device, monkeypatch, pipe):
    monkeypatch.setenv("METELLUS_TC", "1" if pipe == "tcgen05" else "0")
    r = np.random.default_rng(5)
    M, K, N = 512, 256, 384
    ops = Operations()
    ops.from_numpy(r.normal(0, 1, (M, K)).astype(np.float32), "A")
    ops.from_numpy(r.normal(0, 1, (K, N)).astype(np.float32), "B1")
    ops.from_numpy(r.normal(0, 1, (K, N)).astype(np.float32), "B2")
    ops.matmul(a="A", b="B1", out="c1")
    ops.matmul(a="A", b="B2", out="c2")
    ops.elementwise("mul", out="z", operands=("c1", "c2"))
    res = run(ops)
    assert len(res.groups) == 1 and res.groups[0].strategy.value == "diamond_shared"
    if pipe == "tcgen05":
        assert res.groups[0].pipe == "tcgen05"
    r64 = evaluate(ops, np.float64)
    r32 = evaluate(ops, np.float32)
    assert_matmul_close(res.env["z"], r64["z"], r32["z"], what=f"diamond {pipe}")


def _gated(M, K, N, transpose_b=False, seed=0):
    """act(A @ W1 + b1) * (A @ W3): the dual-GEMM epilogue DAG (GELU-tanh gate)."""
    r = np.random.default_rng(seed)
    ops = Operations()
    ops.from_numpy(r.normal(0, 1, (M, K)).astype(np.float32), "A")
    for w in ("W1", "W3"):
        if transpose_b:
            ops.from_numpy(r.normal(0, K ** -0.5, (N, K)).astype(np.float32), w + "t")
            ops.transpose(w + "t", out=w)
        else:
            ops.from_numpy(r.normal(0, K ** -0.5, (K, N)).astype(np.float32), w)
    ops.from_numpy(r.normal(0, 0.02, (1, N)).astype(np.float32), "b1")
    ops.matmul(a="A", b="W1", out="z1")
    ops.elementwise("add", out="z1b", operands=("z1", "b1"), y_broadcast="row")
    ops.elementwise("mul", out="c", operands=("z1b", "z1b"))
    ops.elementwise("mul", out="c3", operands=("c", "z1b"))
    ops.elementwise("mul", out="k", operands=("c3", 0.044715))
    ops.elementwise("add", out="u", operands=("z1b", "k"))
    ops.elementwise("mul", out="v", operands=("u", 0.7978845608))
    ops.elementwise("tanh", out="t", operands=("v",))
    ops.elementwise("add", out="t1", operands=("t", 1.0))
    ops.elementwise("mul", out="hz", operands=("z1b", 0.5))
    ops.elementwise("mul", out="g", operands=("hz", "t1"))
    ops.matmul(a="A", b="W3", out="z3")
    ops.elementwise("mul", out="U", operands=("g", "z3"))
    return ops


@pytest.mark.parametrize("M,K,N,tb", [(256, 256, 512, False), (200, 96, 96, False), (384, 512, 256, True),
                                      (130, 160, 320, True)])
def test_dual_gemm_epilogue(cuda_device, M, K, N, tb):
    ops = _gated(M, K, N, transpose_b=tb, seed=M + N)
    res = run(ops)
    assert [g.strategy.value for g in res.groups] == ["dual_gemm_epilogue"]
    assert res.groups[0].pipe == "tcgen05"
    r64 = evaluate(ops, np.float64)
    r32 = evaluate(ops, np.float32)
    assert_matmul_close(res.env["U"], r64["U"], r32["U"], what=f"dual {M}x{K}x{N} tb={tb}")


@pytest.mark.parametrize("K", [2048, 4096, 8192])
def test_tc_matmul_long_k(cuda_device, K):
    """Long reductions: the per-32 chunk promotion keeps the error at fp32-dot level."""
    ops, out = _mm(256, K, 256, seed=K)
    res = run(ops)
    assert res.groups[0].pipe == "tcgen05"
    r64 = evaluate(ops, np.float64)
    r32 = evaluate(ops, np.float32)
    assert_matmul_close(res.env[out], r64[out], r32[out], what=f"K={K}")


@pytest.mark.parametrize("M,K,N", [(1024, 1024, 1024), (512, 4096, 512), (200, 1000, 320), (256, 520, 384)])
def test_tc_matmul_split_k_pairs(cuda_device, M, K, N):
    """Few output tiles: a two-CTA cluster per tile splits K and combines the halves
    through distributed shared memory (odd k-tile counts and ragged edges included)."""
    ops, out = _mm(M, K, N, bias=True, relu=True, seed=M + K)
    res = run(ops)
    g = res.groups[0]
    assert g.pipe == "tcgen05" and g.cluster_x == 2, (g.pipe, g.cluster_x)
    r64 = evaluate(ops, np.float64)
    r32 = evaluate(ops, np.float32)
    assert_matmul_close(res.env[out], r64[out], r32[out], what=f"split-K {M}x{K}x{N}")


PAIR_CASES = [
    dict(M=2048, K=512, N=2048, bias=True, relu=True),
    dict(M=2100, K=300, N=2016),                    # ragged; the last pair's odd CTA is wholly past M
    dict(M=2048, K=256, N=1000, transpose_b=True),  # K-major B, ragged N
    dict(M=1536, K=384, N=2560, prologue=True),
]


@pytest.mark.parametrize("case", PAIR_CASES, ids=lambda c: "x".join(str(c[k]) for k in "MKN") + "".join(
    k[0] for k, v in c.items() if v is True))
def test_tc_matmul_cta_pairs(cuda_device, case):
    """Many output tiles: 256 x 128 tiles on CTA pairs (cta_group::2 MMAs issued by the
    even CTA, B split between the two CTAs' shared memory)."""
    ops, out = _mm(**case, seed=case["M"] + case["N"])
    res = run(ops)
    g = res.groups[0]
    assert g.pipe == "tcgen05" and g.cluster_x == 2 and g.grid[1] == -(-case["M"] // 256), (g.pipe, g.grid)
    r64 = evaluate(ops, np.float64)
    r32 = evaluate(ops, np.float32)
    assert_matmul_close(res.env[out], r64[out], r32[out], what=f"pair {case}")


@pytest.mark.parametrize("M,K,N,tb", [(2048, 256, 1024, False), (1800, 200, 1088, True)])
def test_dual_gemm_cta_pairs(cuda_device, M, K, N, tb):
    """The dual GEMM on CTA pairs: the even CTA holds W1's tile, the odd W3's."""
    ops = _gated(M, K, N, transpose_b=tb, seed=M + N)
    res = run(ops)
    g = res.groups[0]
    assert g.strategy.value == "dual_gemm_epilogue" and g.cluster_x == 2 and g.grid[1] == -(-M // 256)
    r64 = evaluate(ops, np.float64)
    r32 = evaluate(ops, np.float32)
    assert_matmul_close(res.env["U"], r64["U"], r32["U"], what=f"dual pair {M}x{K}x{N} tb={tb}")
