"""Oracle for residual + RMSNorm (test infrastructure only).

Restates the reference's ``rmsnorm_kernel`` / ``fused_residual_rmsnorm_kernel``
(``src/blackwell_ops/cuda/basic_ops.cu:16-78``) in float32 numpy, in the
kernel's own summation order (one 256-thread block per row):

* ``v = fp32(x) + fp32(residual)`` (``:56``; ``rmsnorm``: ``v = fp32(x)``).
* thread ``t`` sums ``v[k]^2`` for ``k = t, t + 256, ...`` in order (``:55-58``),
  then the block halves: ``s[t] += s[t + h]`` for ``h = 128, 64, ..., 1`` (``:60-66``).
* ``rstd = 1 / sqrt(s[0] / K + eps)`` (``:67``).
* ``out = dt(v * rstd * fp32(w))`` (``:71-74``), the two products rounded in turn.

Every step is an IEEE fp32 operation with its own rounding (no fused
multiply-add), which is what ``bw_residual_rmsnorm`` computes.  The reference
builds with ``--use_fast_math``, which allows contracted and approximate forms
of the same expression.
"""
from __future__ import annotations

import numpy as np

from .numerics import from_f32, to_f32

THREADS = 256


def residual_rmsnorm(x: np.ndarray, residual: np.ndarray | None, w: np.ndarray, eps: float, dtype: str) -> np.ndarray:
    """x, residual [M, K], w [K] in ``dtype``'s oracle representation -> out [M, K] in the same."""
    f32 = np.float32
    v = to_f32(x, dtype)
    if residual is not None:
        v = (v + to_f32(residual, dtype)).astype(f32)
    m, k = v.shape
    sq = (v * v).astype(f32)
    part = np.zeros((m, THREADS), dtype=f32)
    for j in range(0, k, THREADS):
        cols = sq[:, j:j + THREADS]
        part[:, :cols.shape[1]] = (part[:, :cols.shape[1]] + cols).astype(f32)
    h = THREADS // 2
    while h > 0:
        part[:, :h] = (part[:, :h] + part[:, h:2 * h]).astype(f32)
        h //= 2
    mean = (part[:, 0] / f32(k)).astype(f32)
    rstd = (f32(1.0) / np.sqrt((mean + f32(eps)).astype(f32))).astype(f32)
    out = ((v * rstd[:, None]).astype(f32) * to_f32(w, dtype)[None, :]).astype(f32)
    return from_f32(out, dtype)
