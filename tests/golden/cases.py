"""Case tables shared by ``make_golden.py`` and the tests that read its fixtures.

Seeds feed ``oracle.inputs`` (numpy PCG64), so the same tensors are drawn
wherever the tables are read.
"""
from __future__ import annotations

import numpy as np

# name, seed, N, K, dtype
QUANT_CASES = [
    ("ref_test_96x128_f16", 101, 96, 128, "f16"),
    ("ref_test_96x128_bf16", 102, 96, 128, "bf16"),
    ("ref_test_96x128_f32", 103, 96, 128, "f32"),
    ("odd_17x33_f16", 104, 17, 33, "f16"),
    ("odd_3x100_bf16", 105, 3, 100, "bf16"),
    ("one_1x1_f16", 106, 1, 1, "f16"),
    ("wide_2x4099_f16", 107, 2, 4099, "f16"),
    ("cfg1_3072x1024_f16", 1001, 3072, 1024, "f16"),
    ("cfg1_3072x1024_bf16", 1002, 3072, 1024, "bf16"),
    ("cfg1_3072x1024_f32", 1003, 3072, 1024, "f32"),
    ("qwen_q_2048x1024_f16", 2000, 2048, 1024, "f16"),
    ("qwen_k_1024x1024_f16", 2001, 1024, 1024, "f16"),
    ("qwen_v_1024x1024_f16", 2002, 1024, 1024, "f16"),
    ("qwen_o_1024x2048_f16", 2003, 1024, 2048, "f16"),
    ("qwen_gate_3072x1024_f16", 2004, 3072, 1024, "f16"),
    ("qwen_up_3072x1024_f16", 2005, 3072, 1024, "f16"),
    ("qwen_down_1024x3072_f16", 2006, 1024, 3072, "f16"),
    ("llama8b_gate_14336x4096_bf16", 3001, 14336, 4096, "bf16"),
    ("llama8b_down_4096x14336_bf16", 3002, 4096, 14336, "bf16"),
]

# name, dtype — rows built by ``edge_weight``
EDGE_CASES = [
    ("zero_rows_f16", "f16"),
    ("zero_rows_bf16", "bf16"),
    ("zero_rows_f32", "f32"),
    ("subnormal_rows_f16", "f16"),
    ("ties_f16", "f16"),
    ("ties_bf16", "bf16"),
    ("large_f16", "f16"),
    ("single_nonzero_f16", "f16"),
    ("one_col_f16", "f16"),
    ("nonfinite_f16", "f16"),
    ("nonfinite_bf16", "bf16"),
    ("nonfinite_f32", "f32"),
]

# name, seed, M, N, K, x dtype, w dtype
GEMM_CASES = [
    ("ref_test_64x96x128", 201, 64, 96, 128, "f16", "f16"),
    ("cfg1_16x3072x1024", 1001, 16, 3072, 1024, "f16", "f16"),
    ("m1_1x2048x1024", 202, 1, 2048, 1024, "f16", "f16"),
    ("odd_3x40x48", 203, 3, 40, 48, "f16", "f16"),
    ("bf16_32x256x512", 204, 32, 256, 512, "bf16", "bf16"),
]

# name, seed, r, N, K, scaling
LORA_CASES = [
    ("ref_test_r16_96x128", 301, 16, 96, 128, 2.0),
    ("odd_r8_40x72", 302, 8, 40, 72, 0.5),
    ("nonpow2_r16_128x256", 303, 16, 128, 256, 1.5),
    ("r128_256x512", 304, 128, 256, 512, 2.0),
    ("r64_192x320", 305, 64, 192, 320, 2.0),
]


def _to_dtype(f: np.ndarray, dtype: str) -> np.ndarray:
    from oracle.numerics import from_f32

    return from_f32(np.asarray(f, np.float32), dtype)


def edge_weight(name: str, dtype: str) -> np.ndarray:
    """Hand-built weights that reach each branch of the quantiser."""
    rng = np.random.Generator(np.random.PCG64(4242))
    if name.startswith("zero_rows"):
        w = rng.standard_normal((8, 64), dtype=np.float32) * 0.02
        w[[0, 3, 7]] = 0.0
        return _to_dtype(w, dtype)
    if name.startswith("subnormal_rows"):
        # fp16 subnormals: amax/127 underflows to a zero scale -> codes saturate to +-127
        tiny = np.float32(2.0 ** -24)
        w = np.zeros((4, 16), np.float32)
        w[0, :4] = [tiny, -tiny, 0.0, 2 * tiny]
        w[1, :] = tiny * np.arange(16, dtype=np.float32)
        w[2, 5] = -3 * tiny
        w[3, :] = rng.standard_normal(16, dtype=np.float32) * 0.02
        return _to_dtype(w, dtype)
    if name.startswith("ties"):
        # amax 127 -> scale exactly 1 -> quotients land on .5 ties
        row = np.array([127.0, 0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 126.5, -126.5, 3.5, 64.5, -64.5, 0.0, 4.5, 5.5, 6.5],
                       np.float32)
        w = np.stack([row, -row, row * 0.5, np.roll(row, 3)])
        return _to_dtype(w, dtype)
    if name.startswith("large"):
        w = np.array([[65504.0, -65504.0, 1000.0, -0.001], [60000.0, 30000.0, -15000.0, 7.0]], np.float32)
        return _to_dtype(w, dtype)
    if name.startswith("single_nonzero"):
        w = np.zeros((3, 32), np.float32)
        w[0, 7] = -0.75
        w[1, 31] = 1e-3
        w[2, 0] = 3.0
        return _to_dtype(w, dtype)
    if name.startswith("one_col"):
        return _to_dtype(rng.standard_normal((5, 1), dtype=np.float32), dtype)
    if name.startswith("nonfinite"):
        # inf rows (scale inf: finite values -> 0, inf/inf -> NaN -> 0), NaN rows (scale NaN)
        w = rng.standard_normal((6, 24), dtype=np.float32) * 0.02
        w[0, 3] = np.inf
        w[1, 0] = -np.inf
        w[1, 9] = np.inf
        w[2, 5] = np.nan
        w[3, [2, 20]] = [np.nan, np.inf]
        return _to_dtype(w, dtype)
    raise KeyError(name)
