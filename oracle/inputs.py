"""Seeded synthetic inputs (test infrastructure only).

Distributions follow the workload definitions: weights ~ N(0, 0.02), activations
~ N(0, 1), LoRA A ~ N(0, 1/sqrt(K)), LoRA B ~ N(0, 0.01).  numpy's PCG64 stream
is used so the golden-vector script (run where the reference is importable)
and the tests (run anywhere) draw identical tensors from the same seed.
"""
from __future__ import annotations

import math

import numpy as np

from .numerics import BF16, F16, F32, from_f32


def _normal(seed: int, shape, std: float) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(seed))
    return (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)


def weight(seed: int, n: int, k: int, dtype: str = F16, std: float = 0.02) -> np.ndarray:
    return from_f32(_normal(seed, (n, k), std), dtype)


def activations(seed: int, m: int, k: int, dtype: str = F16, std: float = 1.0) -> np.ndarray:
    return from_f32(_normal(seed, (m, k), std), dtype)


def lora_a(seed: int, r: int, k: int) -> np.ndarray:
    return from_f32(_normal(seed, (r, k), 1.0 / math.sqrt(k)), F16)


def lora_b(seed: int, n: int, r: int, std: float = 0.01) -> np.ndarray:
    return from_f32(_normal(seed, (n, r), std), F16)


# Qwen3-0.6B projection shapes (K -> N) of one decoder layer: the workload's
# 7 projections (q, k, v, o, gate, up, down).
QWEN3_06B_PROJ = (
    ("q_proj", 1024, 2048),
    ("k_proj", 1024, 1024),
    ("v_proj", 1024, 1024),
    ("o_proj", 2048, 1024),
    ("gate_proj", 1024, 3072),
    ("up_proj", 1024, 3072),
    ("down_proj", 3072, 1024),
)

__all__ = ["weight", "activations", "lora_a", "lora_b", "QWEN3_06B_PROJ", "F16", "BF16", "F32"]
