"""kotensor_b200 -- B200-native (sm_100a) group-wise INT8/INT4 dequantizing matmul
behind Kotensor's quantized-weight and MatMul operator surface.

The compute lives in libkt_cuda.so (C ABI: include/kt_cuda.h, CUDA sources in
kotensor_b200/csrc/); this package is the host-side mirror of the reference's
Kotlin interface used by tests, benchmarks and Python callers.
"""
from .quantized import Context, MatMul, Quantization, QuantizedLinear, QuantizedTensor  # noqa: F401
from ._lib import KtError, load as load_library, LIB_PATH  # noqa: F401

__all__ = ["Context", "MatMul", "Quantization", "QuantizedLinear", "QuantizedTensor", "KtError",
           "load_library", "LIB_PATH"]
