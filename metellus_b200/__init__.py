"""metellus_b200 — a B200-native (sm_100a) backend for the Metellus fused-program
compiler: the reference's ``Operations`` builder, SSA IR, fusion rules and
``run`` pipeline, with everything below ``KernelGroup`` rendered to CUDA C++,
compiled by NVRTC and launched through the C-ABI library ``libmetellus_cuda.so``."""

from metellus_b200.api.executable import Executable
from metellus_b200.api.run import RunResult, compile_program, run
from metellus_b200.compute.elementwise import BroadcastSpec
from metellus_b200.orchestrator.builder import Operations

__all__ = ["BroadcastSpec", "Executable", "Operations", "RunResult", "compile_program", "run"]
