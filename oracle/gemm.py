"""Oracle for the W8A16 GEMM ``int8_gemm`` (test infrastructure only).

Reference kernel ``src/blackwell_ops/kernels/int8_gemm.py:15-60`` computes, per
output element, an fp32 accumulation of ``x[m,k] * w_int8[n,k]`` (both
up-cast, ``:46,51``; ``tl.dot`` ``:52``), multiplies the fp32 accumulator by
``scale[n]`` (``:54-55``) and rounds once to ``y``'s dtype (= x.dtype, ``:82``,
``:58``).  The reference's own test checks it against dequantise-then-matmul
in fp32 (``src/blackwell_ops/tests/test_int8_gemm.py:17-18``)::

    w_deq = w_int8.float() * scale.unsqueeze(-1)
    ref = x.float() @ w_deq.t()

``reference_fp32`` is exactly that expression; ``exact`` accumulates in float64
and applies the scale after the sum (the reference kernel's order), which is
the value every fp32-accumulating implementation approximates.
"""
from __future__ import annotations

import numpy as np

from .numerics import from_f32, to_f32
from .quant import dequantize


def reference_fp32(x: np.ndarray, x_dtype: str, q: np.ndarray, scale: np.ndarray, s_dtype: str) -> np.ndarray:
    """``x.float() @ (w_int8.float() * scale[:, None]).t()`` in float32 (test_int8_gemm.py:17-18)."""
    return to_f32(x, x_dtype) @ dequantize(q, scale, s_dtype).T


def exact(x: np.ndarray, x_dtype: str, q: np.ndarray, scale: np.ndarray, s_dtype: str) -> np.ndarray:
    """float64 accumulation of x.q, then x scale[n] (int8_gemm.py:52-55 order)."""
    acc = to_f32(x, x_dtype).astype(np.float64) @ q.astype(np.float64).T
    return acc * to_f32(scale, s_dtype).astype(np.float64)[None, :]


def int8_gemm(x: np.ndarray, x_dtype: str, q: np.ndarray, scale: np.ndarray, s_dtype: str) -> np.ndarray:
    """Oracle output in x's dtype representation: dt(fp32(acc) * fp32(scale))."""
    acc = (to_f32(x, x_dtype).astype(np.float64) @ q.astype(np.float64).T).astype(np.float32)
    return from_f32(acc * to_f32(scale, s_dtype)[None, :], x_dtype)


def int8_gemm_swiglu(x: np.ndarray, x_dtype: str, qg: np.ndarray, sg: np.ndarray, qu: np.ndarray, su: np.ndarray,
                     s_dtype: str) -> np.ndarray:
    """``swiglu(int8_gemm(x, w_gate, s_gate), int8_gemm(x, w_up, s_up))`` in x's dtype representation.

    The reference swiglu kernel (src/blackwell_ops/cuda/basic_ops.cu:112-122) up-casts both
    (already dt-rounded) inputs to fp32, computes ``g / (1 + exp(-g)) * u`` in fp32 and rounds once.
    """
    g = to_f32(int8_gemm(x, x_dtype, qg, sg, s_dtype), x_dtype)
    u = to_f32(int8_gemm(x, x_dtype, qu, su, s_dtype), x_dtype)
    with np.errstate(over="ignore"):
        silu = (g / (np.float32(1.0) + np.exp(-g))).astype(np.float32)
    return from_f32((silu * u).astype(np.float32), x_dtype)
