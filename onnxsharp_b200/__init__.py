"""onnxsharp_b200 — B200-native (sm_100a) kernels behind OnnxSharp's matrix-multiply operators.

The compute lives in ``libonnxsharp_cuda.so`` (CUDA C++ for sm_100a, C ABI in
``include/onnxsharp_cuda.h``); this package holds the ctypes binding and the
host-side mirror of the reference's operator interface.
"""
from ._lib import ACT_NONE, ACT_RELU, ACT_SIGMOID, ACT_SILU, OscError, OscUnavailable  # noqa: F401

__all__ = ["OscError", "OscUnavailable", "ACT_NONE", "ACT_SILU", "ACT_RELU", "ACT_SIGMOID"]
