"""ctypes binding of ``libmetellus_cuda.so`` — the replacement for the reference's
nanobind module ``metal_backend`` (src/metal_backend.mm:253-261).

Function names mirror the reference module (``create_buffer``, ``release_buffer``,
``buffer_size``, ``write_buffer``, ``read_buffer``, ``fill_buffer``, ``run_kernel``)
so the runtime layer above reads like the reference's. Errors raise
``RuntimeError`` with the backend's message, as nanobind did.

Differences by design: kernels are compiled once by NVRTC and cached in memory and on
disk (keyed by a SHA-256 of source + options), launches are asynchronous on one
stream per device, and every call names the device explicitly (one process drives
one GPU; the device defaults to ``LOCAL_RANK`` under torchrun).

There is no CPU fallback: importing works anywhere, but the first call that needs the
library raises if ``libmetellus_cuda.so`` is missing, and device calls raise if no GPU
is present.
"""

from __future__ import annotations

import ctypes
import hashlib
import os
import threading
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent.parent
LIB_PATH = PKG / "_lib" / "libmetellus_cuda.so"
ARCH = "sm_100a"
NVRTC_OPTS = f"--gpu-architecture={ARCH} -default-device -std=c++17 -lineinfo -DNDEBUG --diag-suppress=177,550"

_lib: ctypes.CDLL | None = None
_lock = threading.Lock()
_kernel_cache: dict[tuple[str, str], int] = {}
_device = int(os.environ.get("METELLUS_DEVICE", os.environ.get("LOCAL_RANK", "0")))


class MtTmapSpec(ctypes.Structure):
    _fields_ = [
        ("buf_index", ctypes.c_int32),
        ("rank", ctypes.c_uint32),
        ("dims", ctypes.c_uint64 * 5),
        ("strides", ctypes.c_uint64 * 4),
        ("box", ctypes.c_uint32 * 5),
        ("elem_strides", ctypes.c_uint32 * 5),
        ("swizzle", ctypes.c_int32),
        ("l2_promo", ctypes.c_int32),
        ("byte_offset", ctypes.c_uint64),
    ]


EXPORTED = (
    "mt_last_error", "mt_device_count", "mt_init", "mt_device_attr", "mt_buffer_create",
    "mt_buffer_release", "mt_buffer_size", "mt_buffer_ptr", "mt_buffer_write", "mt_buffer_read",
    "mt_buffer_write_async", "mt_buffer_read_async", "mt_buffer_fill", "mt_buffer_fill_async",
    "mt_buffer_read_after", "mt_stream_wait_event", "mt_host_alloc",
    "mt_host_free", "mt_nvrtc_compile", "mt_kernel_load", "mt_kernel_info", "mt_launch", "mt_sync",
    "mt_event_create", "mt_event_record", "mt_event_elapsed", "mt_event_destroy",
    "mt_graph_begin", "mt_graph_end", "mt_graph_launch", "mt_graph_destroy", "mt_reduce_rows",
    "mt_reduce_rows_noalloc", "mt_nccl_unique_id", "mt_nccl_init", "mt_nccl_destroy", "mt_allreduce_f64",
)


def lib() -> ctypes.CDLL:
    """Load the backend library (built by ``metellus_b200.csrc.build``)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"Metellus CUDA backend not built: {LIB_PATH} is missing "
                    "(run `python -m metellus_b200.csrc.build` or __graft_entry__.build())"
                )
            L = ctypes.CDLL(str(LIB_PATH))
            u64, i32, sz = ctypes.c_uint64, ctypes.c_int, ctypes.c_size_t
            P = ctypes.POINTER
            sig = {
                "mt_last_error": [ctypes.c_char_p, sz],
                "mt_device_count": [P(i32)],
                "mt_init": [i32],
                "mt_device_attr": [i32, i32, P(ctypes.c_int64)],
                "mt_buffer_create": [i32, sz, P(u64)],
                "mt_buffer_release": [u64],
                "mt_buffer_size": [u64, P(sz)],
                "mt_buffer_ptr": [u64, P(u64)],
                "mt_buffer_write": [u64, ctypes.c_void_p, sz],
                "mt_buffer_read": [u64, ctypes.c_void_p, sz],
                "mt_buffer_write_async": [u64, ctypes.c_void_p, sz],
                "mt_buffer_read_async": [u64, ctypes.c_void_p, sz],
                "mt_buffer_fill": [u64, ctypes.c_uint8],
                "mt_buffer_fill_async": [u64, ctypes.c_uint8],
                "mt_buffer_read_after": [u64, ctypes.c_void_p, sz, u64, u64],
                "mt_stream_wait_event": [i32, u64],
                "mt_host_alloc": [sz, P(ctypes.c_void_p)],
                "mt_host_free": [ctypes.c_void_p],
                "mt_nvrtc_compile": [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_void_p, sz,
                                     P(sz), ctypes.c_char_p, sz],
                "mt_kernel_load": [ctypes.c_void_p, sz, ctypes.c_char_p, P(u64)],
                "mt_kernel_info": [i32, u64, P(i32), P(i32), P(i32)],
                "mt_launch": [i32, u64, P(u64), i32, P(ctypes.c_uint32), i32, P(ctypes.c_uint32),
                              P(ctypes.c_uint32), ctypes.c_uint32, ctypes.c_uint32, P(MtTmapSpec), i32,
                              P(ctypes.c_float)],
                "mt_sync": [i32],
                "mt_event_create": [P(u64)],
                "mt_event_record": [i32, u64],
                "mt_event_elapsed": [u64, u64, P(ctypes.c_float)],
                "mt_event_destroy": [u64],
                "mt_graph_begin": [i32],
                "mt_graph_end": [i32, P(u64)],
                "mt_graph_launch": [i32, u64],
                "mt_graph_destroy": [u64],
                "mt_reduce_rows": [i32, u64, u64, u64, u64, u64, i32, P(ctypes.c_float)],
                "mt_reduce_rows_noalloc": [i32, ctypes.c_void_p, ctypes.c_void_p, u64, u64, u64, i32,
                                           ctypes.c_void_p],
                "mt_nccl_unique_id": [ctypes.c_char_p, u64],
                "mt_nccl_init": [i32, i32, i32, ctypes.c_char_p],
                "mt_nccl_destroy": [i32],
                "mt_allreduce_f64": [i32, u64, u64, i32, u64],
            }
            for name, args in sig.items():
                fn = getattr(L, name)
                fn.argtypes = args
                fn.restype = ctypes.c_int
            _lib = L
    return _lib


def _check(rc: int) -> None:
    if rc != 0:
        buf = ctypes.create_string_buffer(4096)
        lib().mt_last_error(buf, 4096)
        raise RuntimeError(buf.value.decode(errors="replace"))


# -- devices -----------------------------------------------------------------------


def device_count() -> int:
    n = ctypes.c_int(0)
    _check(lib().mt_device_count(ctypes.byref(n)))
    return n.value


def current_device() -> int:
    return _device


def set_device(dev: int) -> None:
    global _device
    _device = int(dev)


def init(dev: int | None = None) -> None:
    _check(lib().mt_init(_device if dev is None else dev))


def device_attr(which: int, dev: int | None = None) -> int:
    v = ctypes.c_int64(0)
    _check(lib().mt_device_attr(_device if dev is None else dev, which, ctypes.byref(v)))
    return int(v.value)


def sm_count(dev: int | None = None) -> int:
    return device_attr(0, dev)


def max_smem_optin(dev: int | None = None) -> int:
    return device_attr(1, dev)


# -- buffers (reference names: metal_backend.mm:94-141) ----------------------------


def create_buffer(nbytes: int, dev: int | None = None) -> int:
    h = ctypes.c_uint64(0)
    _check(lib().mt_buffer_create(_device if dev is None else dev, int(nbytes), ctypes.byref(h)))
    return int(h.value)


def release_buffer(handle: int) -> bool:
    _check(lib().mt_buffer_release(handle))
    return True


def buffer_size(handle: int) -> int:
    n = ctypes.c_size_t(0)
    _check(lib().mt_buffer_size(handle, ctypes.byref(n)))
    return int(n.value)


def buffer_ptr(handle: int) -> int:
    p = ctypes.c_uint64(0)
    _check(lib().mt_buffer_ptr(handle, ctypes.byref(p)))
    return int(p.value)


def write_buffer(handle: int, array: np.ndarray, *, wait: bool = True) -> None:
    a = np.ascontiguousarray(array)
    fn = lib().mt_buffer_write if wait else lib().mt_buffer_write_async
    _check(fn(handle, a.ctypes.data, a.nbytes))


def read_buffer(handle: int, out: np.ndarray, *, wait: bool = True) -> None:
    if not out.flags["C_CONTIGUOUS"]:
        raise ValueError("read_buffer: destination must be C-contiguous")
    fn = lib().mt_buffer_read if wait else lib().mt_buffer_read_async
    _check(fn(handle, out.ctypes.data, out.nbytes))


def read_buffer_after(handle: int, out: np.ndarray, after: "Event | None" = None,
                      done: "Event | None" = None) -> None:
    """Device-to-host copy on the copy stream after event ``after``; records ``done``."""
    if not out.flags["C_CONTIGUOUS"]:
        raise ValueError("read_buffer_after: destination must be C-contiguous")
    _check(lib().mt_buffer_read_after(handle, out.ctypes.data, out.nbytes, after.handle if after else 0,
                                      done.handle if done else 0))


def stream_wait_event(ev: "Event", dev: int | None = None) -> None:
    _check(lib().mt_stream_wait_event(_device if dev is None else dev, ev.handle))


def fill_buffer(handle: int, value: int, *, wait: bool = True) -> None:
    _check((lib().mt_buffer_fill if wait else lib().mt_buffer_fill_async)(handle, value))


class PinnedArray:
    """Page-locked host array (cudaHostAlloc); ``.array`` is a numpy view of it."""

    def __init__(self, shape: tuple[int, ...], dtype=np.float32) -> None:
        n = int(np.prod(shape)) * np.dtype(dtype).itemsize
        p = ctypes.c_void_p()
        _check(lib().mt_host_alloc(max(n, 1), ctypes.byref(p)))
        self._ptr = p
        buf = (ctypes.c_char * max(n, 1)).from_address(p.value)
        self.array = np.frombuffer(buf, dtype=dtype, count=int(np.prod(shape))).reshape(shape)

    def free(self) -> None:
        if self._ptr is not None:
            lib().mt_host_free(self._ptr)
            self._ptr = None

    def __del__(self) -> None:
        try:
            self.free()
        except Exception:
            pass


def sync(dev: int | None = None) -> None:
    _check(lib().mt_sync(_device if dev is None else dev))


# -- kernels ---------------------------------------------------------------------------


def cache_dir() -> Path:
    d = Path(os.environ.get("METELLUS_CUBIN_CACHE", PKG / "_cubin_cache"))
    d.mkdir(parents=True, exist_ok=True)
    return d


def compile_cubin(source: str, name: str = "kernel.cu", opts: str = NVRTC_OPTS) -> bytes:
    """NVRTC-compile ``source`` to a cubin, through the on-disk cache."""
    key = hashlib.sha256((opts + "\0" + source).encode()).hexdigest()
    path = cache_dir() / f"{key}.cubin"
    if path.exists():
        return path.read_bytes()
    L = lib()
    size = ctypes.c_size_t(0)
    log = ctypes.create_string_buffer(1 << 16)
    _check(L.mt_nvrtc_compile(source.encode(), name.encode(), opts.encode(), None, 0, ctypes.byref(size),
                              log, 1 << 16))
    buf = ctypes.create_string_buffer(size.value)
    _check(L.mt_nvrtc_compile(source.encode(), name.encode(), opts.encode(), buf, size.value,
                              ctypes.byref(size), log, 1 << 16))
    data = buf.raw[: size.value]
    tmp = path.with_suffix(f".tmp{os.getpid()}")
    tmp.write_bytes(data)
    os.replace(tmp, path)
    return data


def load_kernel(source: str, function_name: str) -> int:
    """Compile (cached) and load ``function_name`` from ``source``; returns a handle."""
    ck = (hashlib.sha256(source.encode()).hexdigest(), function_name)
    h = _kernel_cache.get(ck)
    if h is not None:
        return h
    cubin = compile_cubin(source, name=f"{function_name}.cu")
    out = ctypes.c_uint64(0)
    _check(lib().mt_kernel_load(cubin, len(cubin), function_name.encode(), ctypes.byref(out)))
    _kernel_cache[ck] = int(out.value)
    return int(out.value)


def kernel_info(kernel: int, dev: int | None = None) -> dict:
    r, l, t = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0)
    _check(lib().mt_kernel_info(_device if dev is None else dev, kernel, ctypes.byref(r), ctypes.byref(l),
                                ctypes.byref(t)))
    return {"registers": r.value, "local_bytes": l.value, "max_threads": t.value}


def launch(
    kernel: int,
    buffers: list[int] | tuple[int, ...],
    dims: tuple[int, ...],
    grid: tuple[int, int, int],
    threads: tuple[int, int, int],
    *,
    smem: int = 0,
    cluster_x: int = 1,
    tmaps: tuple = (),
    timed: bool = False,
    dev: int | None = None,
) -> float | None:
    """Asynchronous launch on the device stream; with ``timed`` the launch is
    bracketed by events and its device time in ms is returned."""
    nb = len(buffers)
    bufs = (ctypes.c_uint64 * max(nb, 1))(*buffers)
    nd = len(dims)
    dims_arr = (ctypes.c_uint32 * max(nd, 1))(*[int(d) & 0xFFFFFFFF for d in dims])
    g = (ctypes.c_uint32 * 3)(*grid)
    b = (ctypes.c_uint32 * 3)(*threads)
    nt = len(tmaps)
    specs = (MtTmapSpec * max(nt, 1))()
    for i, t in enumerate(tmaps):
        specs[i] = t.to_ctypes()
    ms = ctypes.c_float(0.0)
    _check(lib().mt_launch(_device if dev is None else dev, kernel, bufs, nb, dims_arr, nd, g, b, int(smem),
                           int(cluster_x), specs, nt, ctypes.byref(ms) if timed else None))
    return float(ms.value) if timed else None


class PreparedLaunch:
    """The ctypes argument block of one launch, built once and reused: a dispatch
    replayed many times on the same buffers pays only the ``mt_launch`` call."""

    __slots__ = ("kernel", "bufs", "nb", "dims", "nd", "grid", "block", "smem", "cluster_x", "specs", "nt", "dev")

    def __init__(self, kernel: int, buffers, dims, grid, threads, *, smem: int = 0, cluster_x: int = 1,
                 tmaps: tuple = (), dev: int | None = None) -> None:
        self.kernel = kernel
        self.nb = len(buffers)
        self.bufs = (ctypes.c_uint64 * max(self.nb, 1))(*buffers)
        self.nd = len(dims)
        self.dims = (ctypes.c_uint32 * max(self.nd, 1))(*[int(d) & 0xFFFFFFFF for d in dims])
        self.grid = (ctypes.c_uint32 * 3)(*grid)
        self.block = (ctypes.c_uint32 * 3)(*threads)
        self.smem = int(smem)
        self.cluster_x = int(cluster_x)
        self.nt = len(tmaps)
        self.specs = (MtTmapSpec * max(self.nt, 1))()
        for i, t in enumerate(tmaps):
            self.specs[i] = t.to_ctypes()
        self.dev = _device if dev is None else dev

    def __call__(self, timed: bool = False) -> float | None:
        ms = ctypes.c_float(0.0)
        _check(lib().mt_launch(self.dev, self.kernel, self.bufs, self.nb, self.dims, self.nd, self.grid, self.block,
                               self.smem, self.cluster_x, self.specs, self.nt, ctypes.byref(ms) if timed else None))
        return float(ms.value) if timed else None


def run_kernel(source: str, function_name: str, buffers, grid, threads, *, dims=(), smem: int = 0,
               tmaps=(), cluster_x: int = 1, timed: bool = True) -> dict:
    """Reference-shaped entry (metal_backend.mm:178-249): compile (cached), bind,
    launch and return ``{"time_ms": ...}``."""
    handles = [getattr(x, "handle", x) for x in buffers]
    k = load_kernel(source, function_name)
    t = launch(k, handles, tuple(dims), tuple(grid), tuple(threads), smem=smem, tmaps=tmaps,
               cluster_x=cluster_x, timed=timed)
    return {"time_ms": t if t is not None else 0.0}


REDUCE_OPS = {"sum": 0, "max": 1, "min": 2, "product": 3}
# fp64-output forms (a per-GPU partial of a sharded reduction)
REDUCE_OPS_F64 = {k: v + 4 for k, v in REDUCE_OPS.items()}


def reduce_rows(in_handle: int, out_handle: int, rows: int, cols: int, ld: int, op: str, *,
                timed: bool = False, dev: int | None = None) -> float | None:
    """Native split-row reduction (``mt_reduce_rows``): out[r] = op(in[r, :]); an op
    name ending in ``_f64`` writes fp64 results."""
    ms = ctypes.c_float(0.0)
    code = REDUCE_OPS_F64[op[:-4]] if op.endswith("_f64") else REDUCE_OPS[op]
    _check(lib().mt_reduce_rows(_device if dev is None else dev, in_handle, out_handle, rows, cols, ld,
                                code, ctypes.byref(ms) if timed else None))
    return float(ms.value) if timed else None


# -- NCCL ------------------------------------------------------------------------------

NCCL_ID_BYTES = 128


def nccl_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(NCCL_ID_BYTES)
    _check(lib().mt_nccl_unique_id(buf, NCCL_ID_BYTES))
    return buf.raw


def nccl_init(nranks: int, rank: int, uid: bytes, dev: int | None = None) -> None:
    if len(uid) != NCCL_ID_BYTES:
        raise ValueError(f"NCCL id must be {NCCL_ID_BYTES} bytes, got {len(uid)}")
    _check(lib().mt_nccl_init(_device if dev is None else dev, nranks, rank, uid))


def nccl_destroy(dev: int | None = None) -> None:
    _check(lib().mt_nccl_destroy(_device if dev is None else dev))


def allreduce_f64(buf_handle: int, count: int, op: str = "sum", out_f32: int = 0, dev: int | None = None) -> None:
    """In-place NCCL all-reduce of ``count`` doubles (stream ordered); optionally
    also writes the fp32-rounded result into ``out_f32``."""
    _check(lib().mt_allreduce_f64(_device if dev is None else dev, buf_handle, count, REDUCE_OPS[op], out_f32))


# -- events / graphs -------------------------------------------------------------------


class Event:
    def __init__(self) -> None:
        h = ctypes.c_uint64(0)
        _check(lib().mt_event_create(ctypes.byref(h)))
        self.handle = int(h.value)

    def record(self, dev: int | None = None) -> None:
        _check(lib().mt_event_record(_device if dev is None else dev, self.handle))

    def elapsed_ms(self, end: "Event") -> float:
        ms = ctypes.c_float(0)
        _check(lib().mt_event_elapsed(self.handle, end.handle, ctypes.byref(ms)))
        return float(ms.value)

    def __del__(self) -> None:
        try:
            lib().mt_event_destroy(self.handle)
        except Exception:
            pass


def graph_begin(dev: int | None = None) -> None:
    _check(lib().mt_graph_begin(_device if dev is None else dev))


def graph_end(dev: int | None = None) -> int:
    h = ctypes.c_uint64(0)
    _check(lib().mt_graph_end(_device if dev is None else dev, ctypes.byref(h)))
    return int(h.value)


def graph_launch(graph: int, dev: int | None = None) -> None:
    _check(lib().mt_graph_launch(_device if dev is None else dev, graph))


def graph_destroy(graph: int) -> None:
    _check(lib().mt_graph_destroy(graph))
