"""bybylang_b200 - a B200 (sm_100a) implementation of BybyLang's 4-bit block-quantized
tile-GEMM / GEMV path (OP_TILE_GEMM, micro_kernel/tile_gemm.nim) behind the reference's
`cuda` backend / session operator API.

The kernels live in libbybycuda.so (csrc/, C ABI in include/bybycuda.h); this package is the
host-side mirror of the reference interface over that library.
"""
from . import _lib, distributed, formats, gpubackend, session_vm  # noqa: F401
from ._lib import BybyCudaError  # noqa: F401
from .gpubackend import (GpuBackend, Q4B32Weights, dequant, ensureGpuInit, parseBackend,  # noqa: F401
                         route_for, tile_gemm)
