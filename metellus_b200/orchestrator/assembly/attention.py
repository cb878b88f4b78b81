"""FUSED_ATTENTION strategy (B200): matmul -> [scale] -> row softmax -> matmul in one
kernel. Pattern matching and assembly are added with the attention kernel."""

from __future__ import annotations


def match_attention(graph, blacklist):
    return None


def assemble_attention(decision, function_name):
    raise NotImplementedError("fused attention kernel not built yet")
