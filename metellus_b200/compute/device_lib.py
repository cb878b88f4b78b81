"""Loads the hand-written device headers that NVRTC-compiled kernels include.

The headers live in ``metellus_b200/csrc/include``. Their text is prepended to each
rendered kernel (NVRTC sees no include path), so the cubin cache key — a hash of the
full source — changes whenever a header changes."""

from __future__ import annotations

from pathlib import Path

_INC = Path(__file__).resolve().parent.parent / "csrc" / "include"


def header(name: str) -> str:
    return (_INC / name).read_text()


DEVICE_PRELUDE = header("mt_device.cuh")
