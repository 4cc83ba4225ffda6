"""Oracle for the LoRA delta, merge and requantisation path (test infrastructure only).

``lora_delta`` restates both reference kernels, which compute the same value:

* ``src/blackwell_ops/cuda/lora_ops.cu:16-27`` (one thread per output):
  ``acc += B[n,j] * A[j,k]`` for j = 0..r-1 in fp32, then
  ``delta = __float2half(acc * scaling)``.
* ``src/blackwell_ops/cuda/lora_tiled.cu:20-83`` (64x64 smem tiles): the same
  j-ordered fp32 accumulation (``:63-66``), rounded at ``:79``.

A product of two fp16 values is exact in fp32 (11+11 significant bits), so the
compiler's fused multiply-add and a separate multiply-then-add give the same
bits; the numpy loop below therefore reproduces the reference kernels' fp32
accumulator exactly.

``add_delta`` restates ``src/blackwell_ops/cuda/lora_ops.cu:32-38``:
``W[i] = __float2half(__half2float(W[i]) + __half2float(delta[i]))``.

``merge`` composes the two reference ops (``W' = add_delta_(W, lora_delta(A, B,
s))``); ``merge_requant`` then applies ``quantize_weight_int8``
(``src/blackwell_ops/kernels/int8_gemm.py:63-68``).  The reference LoRA
registry (``src/blackwell_inference/lora/delta_multi.py:59,71,75``) computes
``delta = fp16(fp16(B@A) * scaling)`` and ``W += delta``; for a power-of-two
scaling (alpha = 2r gives 2) it agrees with ``lora_delta`` bit for bit apart
from the fp32 accumulation order inside ``B@A``.
"""
from __future__ import annotations

import numpy as np

from .numerics import F16
from .quant import quantize_weight_int8


def delta_acc(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    """fp32 accumulator of B@A in the reference kernels' j order (exact emulation)."""
    A32 = np.asarray(A, dtype=np.float16).astype(np.float32)
    B32 = np.asarray(B, dtype=np.float16).astype(np.float32)
    r = A32.shape[0]
    acc = np.zeros((B32.shape[0], A32.shape[1]), dtype=np.float32)
    for j in range(r):
        acc += B32[:, j : j + 1] * A32[j : j + 1, :]
    return acc


def delta_exact(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    """float64 B@A (the value every fp32 accumulation order approximates)."""
    return np.asarray(B, np.float64) @ np.asarray(A, np.float64)


def lora_delta(A: np.ndarray, B: np.ndarray, scaling: float = 1.0) -> np.ndarray:
    """``delta = fp16(fp32(acc) * fp32(scaling))`` as np.float16 [N,K]."""
    acc = delta_acc(A, B)
    with np.errstate(over="ignore"):
        return (acc * np.float32(scaling)).astype(np.float16)


def add_delta(W: np.ndarray, D: np.ndarray) -> np.ndarray:
    """``fp16(fp32(W) + fp32(D))`` as a new array (the reference mutates W)."""
    with np.errstate(over="ignore"):
        return (np.asarray(W, np.float16).astype(np.float32) + np.asarray(D, np.float16).astype(np.float32)).astype(np.float16)


def merge(W: np.ndarray, A: np.ndarray, B: np.ndarray, scaling: float) -> np.ndarray:
    """W' = add_delta_(W, lora_delta(A, B, scaling))."""
    return add_delta(W, lora_delta(A, B, scaling))


def merge_requant(W: np.ndarray, A: np.ndarray, B: np.ndarray, scaling: float):
    """(q, scale) = quantize_weight_int8(W') with W' from ``merge``; also returns W'."""
    Wp = merge(W, A, B, scaling)
    q, s = quantize_weight_int8(Wp, F16)
    return q, s, Wp


def registry_delta(A: np.ndarray, B: np.ndarray, scaling: float) -> np.ndarray:
    """``(B @ A) * scaling`` in fp16 as the reference registry does it (delta_multi.py:59)."""
    acc = delta_exact(A, B).astype(np.float32).astype(np.float16)
    with np.errstate(over="ignore"):
        return (acc.astype(np.float32) * np.float32(scaling)).astype(np.float16)
