"""sharpinfer_b200: B200 (sm_100a) K-quant hot path for SharpInfer.

The compute lives in libsharpinfer_b200.so (CUDA kernels behind a C ABI,
include/sharpinfer_b200.h).  This package is the host-side binding used by the
tests and the benchmark; `backend` mirrors SharpInfer's IComputeBackend.
"""
from . import native  # noqa: F401
from .backend import B200Context, QuantWeight  # noqa: F401
