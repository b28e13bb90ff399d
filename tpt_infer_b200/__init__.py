"""tpt_infer_b200 -- a B200-native (sm_100a) CUDA backend for tpt-infer.

The product is ``libtpt_cuda.so`` (C ABI: include/tpt_cuda.h), hand-written
CUDA kernels for the dense contractions of tpt-infer's Backend HAL and its
INT8/INT4 quantized-weight path. This package holds the build recipe and a
Python mirror of the reference interfaces (``CudaBackend`` for the Backend
trait, plus the tpt-infer-quantize entry points) used by the tests and the
benchmark. There is no CPU fallback: without the built library the import
fails.
"""
from .backend import (ACT_GELU, ACT_NONE, ACT_RELU, Conv2dOptions, CudaBackend, OpError, Weights)

__all__ = ["CudaBackend", "Conv2dOptions", "OpError", "Weights", "ACT_NONE", "ACT_RELU", "ACT_GELU"]
