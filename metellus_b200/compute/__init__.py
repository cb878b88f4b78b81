"""CUDA C++ fragment library: elementwise op tables, tile copies, matmul tiles,
reductions and strided copies, each rendered into NVRTC-compiled kernels."""
