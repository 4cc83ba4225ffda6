"""B200 kernels with the reference's names (``src/blackwell_ops/kernels/__init__.py:1``), plus the
fused gate/up + SwiGLU GEMM (``int8_gemm_swiglu``), the RMSNorm-prologue GEMM (``int8_gemm_rmsnorm``)
and the grouped GEMM over projections sharing an input (``int8_gemm_grouped``)."""
from .int8_gemm import int8_gemm, int8_gemm_grouped, int8_gemm_rmsnorm, int8_gemm_swiglu, quantize_weight_int8

__all__ = ["int8_gemm", "int8_gemm_grouped", "int8_gemm_rmsnorm", "int8_gemm_swiglu", "quantize_weight_int8"]
