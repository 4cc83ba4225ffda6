"""CPU checks of the residual + RMSNorm oracle (oracle/norm.py).

Against the reference test's own expression (src/blackwell_ops/tests/test_cuda_basic.py:21-30:
``x_f = (x + r).float(); x_f / sqrt(mean(x_f^2) + 1e-6) * w``, tolerance 0.01) and against a
float64 evaluation of the same formula (the restatement's summation order moves the result by
no more than a few fp16 units in the last place).
"""
import numpy as np

from oracle import norm
from oracle.numerics import BF16, F16, from_f32, to_f32


def _case(seed, m, k, dt):
    rng = np.random.Generator(np.random.PCG64(seed))
    mk = lambda shape: from_f32(rng.standard_normal(shape, dtype=np.float32), dt)  # noqa: E731
    return mk((m, k)), mk((m, k)), mk((k,))


def test_matches_the_reference_test_expression():
    x, r, w = _case(1, 64, 512, F16)
    out = to_f32(norm.residual_rmsnorm(x, r, w, 1e-6, F16), F16)
    xf = (x + r).astype(np.float32)  # the test adds in fp16, then widens
    ref = xf / np.sqrt((xf * xf).mean(axis=-1, keepdims=True) + 1e-6) * w.astype(np.float32)
    assert np.abs(out - ref).max() < 0.01


def test_close_to_float64_formula():
    for dt, k in ((F16, 4096), (BF16, 3000), (F16, 1), (BF16, 257)):
        x, r, w = _case(k, 8, k, dt)
        out = to_f32(norm.residual_rmsnorm(x, r, w, 1e-6, dt), dt).astype(np.float64)
        v = to_f32(x, dt).astype(np.float64) + to_f32(r, dt).astype(np.float64)
        ref = v / np.sqrt((v * v).mean(axis=-1, keepdims=True) + 1e-6) * to_f32(w, dt).astype(np.float64)
        ulp = 2.0 ** -10 if dt == F16 else 2.0 ** -7
        assert (np.abs(out - ref) <= 2 * ulp * np.abs(ref) + 1e-6).all()


def test_plain_rmsnorm_is_the_residual_free_case():
    x, _, w = _case(3, 4, 1000, F16)
    zeros = np.zeros_like(x)
    a = norm.residual_rmsnorm(x, None, w, 1e-6, F16)
    b = norm.residual_rmsnorm(x, zeros, w, 1e-6, F16)
    assert np.array_equal(a.view(np.uint16), b.view(np.uint16))
