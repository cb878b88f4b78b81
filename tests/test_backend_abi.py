"""CPU checks of the C-ABI library: it loads without a GPU and exports every entry
point declared in include/metellus_b200.h; error paths report through mt_last_error.
No compute calls are made here."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from metellus_b200.runtime import backend

HEADER = Path(__file__).resolve().parents[1] / "include" / "metellus_b200.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*int\s+(mt_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_binding_set():
    assert declared_symbols() == sorted(backend.EXPORTED)


def test_library_exports_every_declared_symbol():
    lib = backend.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_unknown_handle_raises_runtime_error():
    with pytest.raises(RuntimeError, match="unknown buffer handle"):
        backend.buffer_size(123456789)


def test_nvrtc_compile_error_surfaces_log():
    with pytest.raises(RuntimeError, match="NVRTC compile"):
        backend.compile_cubin('extern "C" __global__ void k() { this is not cuda; }', name="bad.cu")


def test_last_error_is_thread_local_string():
    buf = ctypes.create_string_buffer(256)
    assert backend.lib().mt_last_error(buf, 256) == 0
