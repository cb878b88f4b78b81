"""Host runtime: buffers, runtime steps and the ctypes backend binding."""

from metellus_b200.runtime.buffer import Buffer
from metellus_b200.runtime.program import (
    Allocate,
    Dispatch,
    Download,
    Env,
    Fill,
    Free,
    FromNumpy,
    Kernel,
    Runtime,
    RuntimeFragment,
    Upload,
)

__all__ = ["Allocate", "Buffer", "Dispatch", "Download", "Env", "Fill", "Free", "FromNumpy",
           "Kernel", "Runtime", "RuntimeFragment", "Upload"]
