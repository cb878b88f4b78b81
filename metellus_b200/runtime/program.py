"""Host-side runtime steps (reference: src/runtime/program.py:27-215).

``Runtime`` is an ordered list of steps run against an env dict: ``FromNumpy`` /
``Allocate`` / ``Free`` / ``Upload`` / ``Download`` / ``Fill`` manage buffers,
``Kernel`` renders (and here also compiles) a kernel, ``Dispatch`` launches it.

CUDA differences: ``Kernel.execute`` compiles through NVRTC and the cubin cache off
the hot path (the reference's Metal backend recompiled on every ``run_kernel``,
metal_backend.mm:191); ``Dispatch`` passes dims by value instead of allocating a dims
buffer per launch (program.py:186) and launches asynchronously — only ``Download``,
profile timing and explicit syncs wait for the device.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Protocol

import numpy as np

from metellus_b200.compute.fragments import CodegenContext, CodegenEngine, smem_bytes_of
from metellus_b200.runtime import backend
from metellus_b200.runtime.buffer import Buffer

Env = dict[str, Any]


class RuntimeFragment(Protocol):
    def execute(self, env: Env) -> None: ...


@dataclass(frozen=True)
class Allocate:
    name: str
    nbytes: int

    def execute(self, env: Env) -> None:
        if self.name in env:
            raise KeyError(f"Allocate: key {self.name!r} already in env")
        env[self.name] = Buffer(self.nbytes)


@dataclass(frozen=True)
class Free:
    name: str

    def execute(self, env: Env) -> None:
        env.pop(self.name).release()


@dataclass(frozen=True)
class Upload:
    name: str
    source: np.ndarray

    def execute(self, env: Env) -> None:
        env[self.name].write(self.source)


@dataclass(frozen=True)
class FromNumpy:
    name: str
    source: np.ndarray

    def execute(self, env: Env) -> None:
        if self.name in env:
            raise KeyError(f"FromNumpy: key {self.name!r} already in env")
        env[self.name] = Buffer.from_numpy(self.source)


@dataclass(frozen=True)
class Download:
    """Read a buffer into a fresh ndarray at env[into]; with strides, gather a view
    host-side (program.py:288-335)."""

    name: str
    shape: tuple[int, ...]
    dtype: Any
    into: str
    row_stride: int | None = None
    col_stride: int | None = None
    batch_stride: int | None = None

    def execute(self, env: Env) -> None:
        buf = env[self.name]
        if self.row_stride is None:
            env[self.into] = buf.numpy(self.shape, self.dtype)
            return
        item = np.dtype(self.dtype).itemsize
        flat = buf.numpy((buf.nbytes // item,), self.dtype)
        if len(self.shape) == 3:
            st = ((self.batch_stride or 0) * item, self.row_stride * item, (self.col_stride or 0) * item)
        elif len(self.shape) == 2:
            st = (self.row_stride * item, (self.col_stride or 0) * item)
        elif len(self.shape) == 1:
            st = (self.row_stride * item,)
        else:
            raise ValueError(f"Download with strides supports 1D..3D shapes; got {self.shape}")
        view = np.lib.stride_tricks.as_strided(flat, shape=self.shape, strides=st, writeable=False)
        env[self.into] = np.ascontiguousarray(view)


@dataclass(frozen=True)
class TmapSpec:
    """A TMA tensor map the backend encodes at launch (fp32 elements).

    ``buf_index`` indexes the launch's buffer list; ``dims`` / ``box`` are innermost
    first, ``strides`` are byte strides of dims 1.. ; ``swizzle`` 0/1/2/3 = none /
    32B / 64B / 128B."""

    buf_index: int
    dims: tuple[int, ...]
    strides: tuple[int, ...]
    box: tuple[int, ...]
    swizzle: int = 3
    l2_promo: int = 2

    def to_ctypes(self):
        s = backend.MtTmapSpec()
        s.buf_index = self.buf_index
        s.rank = len(self.dims)
        for i, d in enumerate(self.dims):
            s.dims[i] = d
            s.box[i] = self.box[i]
            s.elem_strides[i] = 1
        for i, st in enumerate(self.strides):
            s.strides[i] = st
        s.swizzle = self.swizzle
        s.l2_promo = self.l2_promo
        s.byte_offset = 0
        return s


@dataclass(frozen=True)
class CheckStatus:
    """Read a kernel status word; nonzero means a bounded wait in a kernel timed out
    (the kernel returned early and its outputs are invalid)."""

    name: str

    def execute(self, env: Env) -> None:
        buf = env.get(self.name)
        if buf is None:
            return
        words = buf.numpy((buf.nbytes // 4,), np.int32)
        if words.any():
            raise RuntimeError(
                f"kernel status {words[:4].tolist()}: a device-side wait timed out "
                "(1=producer, 2=mma, 3=converter, 4=softmax, 5=accumulator, 6/7=split-K exchange); "
                "results are invalid"
            )


@dataclass(frozen=True)
class Fill:
    name: str
    byte_value: int = 0

    def execute(self, env: Env) -> None:
        env[self.name].fill(self.byte_value)


class Kernel:
    """A rendered, lazily compiled CUDA kernel (program.py:126-161)."""

    def __init__(self, fragments: tuple[Any, ...], ctx: CodegenContext) -> None:
        self.fragments = tuple(fragments)
        self.ctx = ctx
        self._source: str | None = None
        self._handle: int | None = None
        self._dims_slot_index = ctx.dims_buffer_index if ctx.dims_buffer_index is not None else len(ctx.buffers)

    @property
    def source(self) -> str:
        if self._source is None:
            self._source = CodegenEngine().render(list(self.fragments), self.ctx)
        return self._source

    @property
    def function_name(self) -> str:
        return self.ctx.function_name

    @property
    def dims_slot_index(self) -> int:
        return self._dims_slot_index

    @property
    def dim_names(self) -> tuple[str, ...]:
        return self.ctx.dims

    @property
    def smem_bytes(self) -> int:
        """Dynamic shared memory the launch needs (arena of all tile decls)."""
        return smem_bytes_of(self.ctx)

    @property
    def handle(self) -> int:
        if self._handle is None:
            self._handle = backend.load_kernel(self.source, self.function_name)
        return self._handle

    def execute(self, env: Env) -> None:
        _ = self.handle


class NativeKernel(Kernel):
    """A kernel compiled ahead of time into ``libmetellus_cuda.so`` and launched
    through its own C-ABI entry point (no NVRTC source). ``entry`` names the
    backend function; ``params`` its static arguments."""

    def __init__(self, entry: str, params: tuple, ctx: CodegenContext) -> None:
        super().__init__(fragments=(), ctx=ctx)
        self.entry = entry
        self.params = tuple(params)

    @property
    def source(self) -> str:
        return f"// native kernel {self.entry}{self.params}\n"

    @property
    def smem_bytes(self) -> int:
        return 0

    @property
    def handle(self) -> int:
        return 0

    def launch(self, handles: list[int], timed: bool) -> float | None:
        if self.entry == "mt_reduce_rows":
            rows, cols, ld, op = self.params
            return backend.reduce_rows(handles[0], handles[1], rows, cols, ld, op, timed=timed)
        if self.entry == "mt_reduce_rows+mt_allreduce_f64":
            # handles: input, output, fp64 partial scratch
            rows, cols, ld, op = self.params
            t0 = backend.Event() if timed else None
            if t0 is not None:
                t0.record()
            backend.reduce_rows(handles[0], handles[2], rows, cols, ld, op + "_f64")
            backend.allreduce_f64(handles[2], rows, op, out_f32=handles[1])
            if t0 is None:
                return None
            t1 = backend.Event()
            t1.record()
            backend.sync()
            return t0.elapsed_ms(t1)
        raise ValueError(f"unknown native kernel {self.entry!r}")


@dataclass(frozen=True)
class Dispatch:
    """Launch a Kernel with env buffers in binding order (program.py:164-197)."""

    kernel: Kernel
    bindings: tuple[str, ...]
    dims: tuple[int, ...]
    grid: tuple[int, int, int]
    threads: tuple[int, int, int]
    time_key: str | None = None
    tmaps: tuple = ()
    cluster_x: int = 1

    def execute(self, env: Env) -> None:
        if len(self.dims) != len(self.kernel.dim_names):
            raise ValueError(
                f"Dispatch: expected {len(self.kernel.dim_names)} dim values "
                f"({self.kernel.dim_names}), got {len(self.dims)}"
            )
        handles = tuple(env[name].handle for name in self.bindings)
        if isinstance(self.kernel, NativeKernel):
            t = self.kernel.launch(list(handles), self.time_key is not None)
            if self.time_key is not None:
                env[self.time_key] = float(t)
            return
        # the argument block is rebuilt only when the bound buffers change
        cached = self.__dict__.get("_prepared")
        if cached is None or cached[0] != (handles, backend.current_device()):
            prep = backend.PreparedLaunch(self.kernel.handle, handles, self.dims, self.grid, self.threads,
                                          smem=self.kernel.smem_bytes, tmaps=self.tmaps, cluster_x=self.cluster_x)
            cached = ((handles, backend.current_device()), prep)
            object.__setattr__(self, "_prepared", cached)
        t = cached[1](timed=self.time_key is not None)
        if self.time_key is not None:
            env[self.time_key] = float(t)


@dataclass(frozen=True)
class Runtime:
    fragments: tuple[RuntimeFragment, ...] = field(default_factory=tuple)

    def run(self, env: Env | None = None) -> Env:
        if env is None:
            env = {}
        for f in self.fragments:
            f.execute(env)
        return env

    def __add__(self, other: "Runtime") -> "Runtime":
        return Runtime(self.fragments + other.fragments)
