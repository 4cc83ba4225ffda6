"""Oracle for the KV-cache per-channel int8 quantiser (test infrastructure only).

Restates the reference's ``quantize_per_channel_kernel`` /
``dequantize_per_channel_kernel`` (``src/blackwell_ops/cuda/kv_quant.cu:17-58``)
in float32 numpy, with the source's arithmetic (IEEE fp32):

* ``amax``  = max over the channel of ``fabsf(float(x))`` with ``fmaxf``
  (``:26-35``): NaN elements never win a comparison, the running maximum
  starts at 0, so a row of zeros and NaNs has ``amax`` 0.
* ``scale`` = ``amax / 127.0f`` in fp32, stored as fp32 (``:36-37``).
* ``q``     = ``clamp((int)lrintf(float(x) / scale), -127, 127)`` (``:40-41``):
  fp32 quotient, round half to even; a NaN quotient (0/0, NaN input,
  inf/inf) converts to 0.  A finite non-zero scale bounds every quotient by
  127.0000x, so the clamp never meets an infinite quotient.
* dequantise: ``x' = __float2half(float(q) * scale)`` (``:55``), fp32 product
  rounded once to fp16.

The reference builds its extension with ``--use_fast_math`` (its loader,
``src/blackwell_ops/cuda/__init__.py:52-55``), which lets the compiler
replace the two divisions with approximate ones; the source's own arithmetic
(restated here and implemented by ``bw_quantize_kv_int8``) is IEEE.
"""
from __future__ import annotations

import numpy as np


def quantize_kv_int8(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """x [C, N] float16 -> (q [C, N] int8, scale [C] float32)."""
    f = np.asarray(x, dtype=np.float16).astype(np.float32)
    if f.shape[1] == 0:
        amax = np.zeros(f.shape[0], dtype=np.float32)
    else:
        amax = np.fmax.reduce(np.abs(f), axis=1, initial=np.float32(0.0)).astype(np.float32)
    scale = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        v = (f / scale[:, None]).astype(np.float32)
    r = np.rint(v)
    r[np.isnan(r)] = 0.0
    q = np.clip(r, -127, 127).astype(np.int8)
    return q, scale


def dequantize_kv_int8(q: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """q [C, N] int8, scale [C] float32 -> x [C, N] float16.

    A NaN product (code 0 times an inf scale) converts to CUDA's fp16 NaN,
    0x7FFF, as ``__float2half`` does (numpy would give 0x7E00)."""
    with np.errstate(invalid="ignore"):
        prod = (np.asarray(q).astype(np.float32) * np.asarray(scale, dtype=np.float32)[:, None]).astype(np.float32)
    out = prod.astype(np.float16)
    out.view(np.uint16)[np.isnan(prod)] = 0x7FFF
    return out
