"""Owning handle to a device buffer (reference: src/runtime/buffer.py:8-91).

Same surface: ``Buffer(nbytes)``, ``from_numpy``, ``zeros``, ``handle``, ``nbytes``,
``write``, ``read_into``, ``numpy``, ``fill``, ``release`` and release on ``__del__``.
Backed by the stream-ordered pool of ``libmetellus_cuda.so`` on one device."""

from __future__ import annotations

import numpy as np

from metellus_b200.runtime import backend


class Buffer:
    __slots__ = ("_handle", "_nbytes", "_released", "_device")

    def __init__(self, nbytes: int, device: int | None = None) -> None:
        if nbytes <= 0:
            raise ValueError(f"Buffer nbytes must be > 0; got {nbytes}")
        self._device = backend.current_device() if device is None else device
        self._handle = backend.create_buffer(nbytes, self._device)
        self._nbytes = nbytes
        self._released = False

    @classmethod
    def from_numpy(cls, array: np.ndarray, device: int | None = None) -> "Buffer":
        a = np.ascontiguousarray(array)
        buf = cls(a.nbytes, device)
        backend.write_buffer(buf._handle, a)
        return buf

    @classmethod
    def zeros(cls, nbytes: int, device: int | None = None) -> "Buffer":
        buf = cls(nbytes, device)
        backend.fill_buffer(buf._handle, 0)
        return buf

    @property
    def handle(self) -> int:
        if self._released:
            raise RuntimeError("Buffer has been released")
        return self._handle

    @property
    def nbytes(self) -> int:
        return self._nbytes

    @property
    def device(self) -> int:
        return self._device

    def write(self, array: np.ndarray, *, wait: bool = True) -> None:
        a = np.ascontiguousarray(array)
        if a.nbytes > self._nbytes:
            raise ValueError(f"write: source ({a.nbytes} bytes) exceeds buffer ({self._nbytes} bytes)")
        backend.write_buffer(self.handle, a, wait=wait)

    def read_into(self, out: np.ndarray, *, wait: bool = True) -> np.ndarray:
        if not out.flags["C_CONTIGUOUS"]:
            raise ValueError("read_into: destination must be C-contiguous")
        if out.nbytes > self._nbytes:
            raise ValueError(f"read_into: destination ({out.nbytes} bytes) exceeds buffer ({self._nbytes} bytes)")
        backend.read_buffer(self.handle, out, wait=wait)
        return out

    def numpy(self, shape: tuple[int, ...], dtype=np.float32) -> np.ndarray:
        return self.read_into(np.empty(shape, dtype=dtype))

    def fill(self, byte_value: int) -> None:
        if not 0 <= byte_value <= 255:
            raise ValueError(f"fill byte_value must be in [0, 255]; got {byte_value}")
        backend.fill_buffer(self.handle, byte_value)

    def release(self) -> None:
        if not self._released:
            backend.release_buffer(self._handle)
            self._released = True

    def __del__(self) -> None:
        try:
            self.release()
        except Exception:
            pass

    def __repr__(self) -> str:
        state = "released" if self._released else f"handle={self._handle}"
        return f"Buffer(nbytes={self._nbytes}, device={self._device}, {state})"
