"""tcgen05 / TMEM 3xTF32 matmul path (B200). Until it is wired in, every matmul
group takes the SIMT FFMA pipe."""

from __future__ import annotations


def try_assemble_tc_matmul(decision, function_name):
    return None


def try_assemble_tc_multi_anchor(decision, function_name):
    return None
