"""cuda_inf_b200: B200-native (sm_100a) quantized decode hot path of g023/cuda_inf.

libcuinf.so (csrc/) holds the CUDA kernels, the C ABI (include/cuinf.h) and
the C++ decode engine; this package is the Python side of that ABI:
  ops      reference-named operators on torch CUDA tensors
  weights  the weights.bin/index.bin format (writer, synthetic models)
  engine   Model / Session (CUDA-graph decode step)
"""
from ._lib import CuinfConfig, CuinfError, lib  # noqa: F401

__version__ = "0.1.0"
