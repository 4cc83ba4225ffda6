"""CPU: the oracle of the fused gate/up + SwiGLU op against an independent
float64 statement of the reference composition (int8_gemm twice, then the
reference swiglu kernel's fp32 ``g / (1 + exp(-g)) * u``, basic_ops.cu:112-122)."""
import numpy as np

from oracle import gemm, inputs, quant
from oracle.numerics import BF16, F16, to_f32


def test_swiglu_oracle_matches_float64_composition():
    for dt in (F16, BF16):
        x = inputs.activations(3, 5, 96, dt)
        qg, sg = quant.quantize_weight_int8(inputs.weight(4, 40, 96, dt), dt)
        qu, su = quant.quantize_weight_int8(inputs.weight(5, 40, 96, dt), dt)
        y = to_f32(gemm.int8_gemm_swiglu(x, dt, qg, sg, qu, su, dt), dt).astype(np.float64)
        g = to_f32(gemm.int8_gemm(x, dt, qg, sg, dt), dt).astype(np.float64)
        u = to_f32(gemm.int8_gemm(x, dt, qu, su, dt), dt).astype(np.float64)
        want = g / (1.0 + np.exp(-g)) * u
        ulp = 2.0 ** -10 if dt == F16 else 2.0 ** -7
        assert np.all(np.abs(y - want) <= ulp * np.abs(want) + 1e-6)
