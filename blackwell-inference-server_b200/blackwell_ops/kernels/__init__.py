"""B200 kernels with the reference's names (``src/blackwell_ops/kernels/__init__.py:1``)."""
from .int8_gemm import int8_gemm, quantize_weight_int8

__all__ = ["int8_gemm", "quantize_weight_int8"]
