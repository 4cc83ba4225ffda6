"""Oracle for per-output-channel symmetric int8 quantisation (test infrastructure only).

Restates ``quantize_weight_int8`` from the reference,
``src/blackwell_ops/kernels/int8_gemm.py:63-68``::

    w_abs_max = w.abs().amax(dim=-1, keepdim=True).clamp(min=1e-8)   # :65
    scale = w_abs_max / 127.0                                        # :66
    w_int8 = (w / scale).round().clamp(-127, 127).to(torch.int8)     # :67

with every intermediate rounded the way torch rounds it (``dt`` = the
weight's dtype; fp16/bf16 arithmetic is done in fp32 and rounded back):

* ``amax``  = max |w| over the row, exact in ``dt``; NaN propagates.
* ``amax_c``= dt(max(fp32(amax), fp32(1e-8)))   (fp16: 1e-8 rounds to 0).
* ``scale`` = dt(fp32(amax_c) / 127.0f)          IEEE division.
* ``x``     = dt(fp32(w) / fp32(scale))          rounded to dt BEFORE rounding
                                                 to an integer.
* ``q``     = clamp(rint(x), -127, 127) as int8; NaN -> 0 (torch's NaN ->
              int8 cast on CPU), +-inf -> +-127 (clamped first).

The ``dt`` rounding of the quotient is load-bearing: dropping it changes tens
of thousands of codes at the 3072x1024 shape.
"""
from __future__ import annotations

import numpy as np

from .numerics import F32, from_f32, round_to, to_f32


def row_scale(w: np.ndarray, dtype: str) -> np.ndarray:
    """Per-row scale as float32 values that are exactly representable in ``dtype``."""
    f = to_f32(w, dtype)
    amax = np.max(np.abs(f), axis=-1) if f.shape[-1] else np.zeros(f.shape[:-1], np.float32)
    amax_c = round_to(np.maximum(amax, np.float32(1e-8)), dtype)
    with np.errstate(divide="ignore", invalid="ignore"):
        return round_to(amax_c / np.float32(127.0), dtype)


def quantize_codes(f: np.ndarray, scale_f32: np.ndarray, dtype: str) -> np.ndarray:
    """int8 codes of float32 values ``f`` [N,K] under per-row ``scale_f32`` [N]."""
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        x = round_to(f / scale_f32[:, None], dtype)
        r = np.rint(x)
    nan = np.isnan(r)
    r = np.clip(np.where(nan, 0.0, r), -127.0, 127.0)
    return r.astype(np.int8)


def quantize_weight_int8(w: np.ndarray, dtype: str):
    """Returns ``(q int8 [N,K], scale [N] in dtype's oracle representation)``.

    ``w`` is ``np.float16`` for fp16, uint16 bit patterns for bf16, float32 for
    fp32.  The scale comes back in the same representation.
    """
    scale = row_scale(w, dtype)
    q = quantize_codes(to_f32(w, dtype), scale, dtype)
    return q, from_f32(scale, dtype) if dtype != F32 else scale.astype(np.float32)


def dequantize(q: np.ndarray, scale: np.ndarray, dtype: str) -> np.ndarray:
    """``w_int8.float() * scale.unsqueeze(-1)`` (reference test_int8_gemm.py:17), float32."""
    return q.astype(np.float32) * to_f32(scale, dtype)[:, None]
