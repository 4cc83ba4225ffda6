"""Pin the CPU oracle to the reference's own outputs (golden vectors).

The fixtures were produced by ``tests/golden/make_golden.py`` from the real
reference ``quantize_weight_int8`` and the reference tests' CPU expressions.
"""
import hashlib

import numpy as np
import pytest

from cases import EDGE_CASES, GEMM_CASES, LORA_CASES, QUANT_CASES, edge_weight
from oracle import gemm, inputs, lora, quant
from oracle.numerics import BF16, F16, F32, to_f32


def same_bits(a, b) -> bool:
    """Equal shape, dtype and bytes (NaN compares equal to the same NaN)."""
    a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
    return a.shape == b.shape and a.dtype == b.dtype and a.tobytes() == b.tobytes()


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("case", QUANT_CASES, ids=[c[0] for c in QUANT_CASES])
def test_quantizer_matches_reference_bits(case, golden):
    name, seed, n, k, dt = case
    if n * k > 16_000_000:
        pytest.skip("covered by the GPU full-size test; too slow for the CPU suite")
    data, index = golden
    w = inputs.weight(seed, n, k, dt)
    q, s = quant.quantize_weight_int8(w, dt)
    ent = index["quant"][name]
    assert sha(q) == ent["q_sha256"]
    assert sha(s) == ent["scale_sha256"]


@pytest.mark.parametrize("case", EDGE_CASES, ids=[c[0] for c in EDGE_CASES])
def test_quantizer_edge_cases(case, golden):
    name, dt = case
    data, _ = golden
    w = edge_weight(name, dt)
    assert same_bits(w, data[f"edge/{name}/w"])
    q, s = quant.quantize_weight_int8(w, dt)
    assert np.array_equal(q, data[f"edge/{name}/q"])
    assert same_bits(s, data[f"edge/{name}/scale"])  # NaN scales included


def test_quantizer_dt_rounding_is_load_bearing():
    """Dropping the quotient's rounding to dt changes codes (the plant goes in the oracle)."""
    w = inputs.weight(1001, 3072, 1024, F16)
    q, s = quant.quantize_weight_int8(w, F16)
    f = to_f32(w, F16)
    with np.errstate(divide="ignore", invalid="ignore"):
        wrong = np.clip(np.rint(f / to_f32(s, F16)[:, None]), -127, 127).astype(np.int8)
    assert (wrong != q).sum() > 1000


@pytest.mark.parametrize("case", GEMM_CASES, ids=[c[0] for c in GEMM_CASES])
def test_gemm_oracle_matches_reference_expression(case, golden):
    name, seed, m, n, k, xdt, wdt = case
    data, index = golden
    x = inputs.activations(seed + 1, m, k, xdt)
    w = inputs.weight(seed, n, k, wdt)
    q, s = quant.quantize_weight_int8(w, wdt)
    assert sha(q) == index["gemm"][name]["q_sha256"]
    ref = data[f"gemm/{name}/ref_fp32"]
    mine = gemm.reference_fp32(x, xdt, q, s, wdt)
    np.testing.assert_allclose(mine, ref, rtol=1e-5, atol=1e-5)
    ex = gemm.exact(x, xdt, q, s, wdt)
    np.testing.assert_allclose(ex, ref, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("case", LORA_CASES, ids=[c[0] for c in LORA_CASES])
def test_lora_oracle_matches_reference_expressions(case, golden):
    name, seed, r, n, k, scaling = case
    data, index = golden
    ent = index["lora"][name]
    A = inputs.lora_a(seed, r, k)
    B = inputs.lora_b(seed + 1, n, r)
    W = inputs.weight(seed + 2, n, k, F16)
    d = lora.lora_delta(A, B, scaling)
    ref32 = data[f"lora/{name}/delta_fp32"]
    rows = ref32.shape[0]
    exact = (lora.delta_exact(A, B) * scaling)[:rows]
    # reference test tolerance (test_lora_ops.py:15) and a much tighter bound
    assert np.abs(d[:rows].astype(np.float32) - ref32).max() < 0.02
    np.testing.assert_allclose(ref32, exact, rtol=1e-5, atol=1e-6)
    ulp = np.spacing(np.abs(d[:rows]).astype(np.float16)).astype(np.float32)
    assert (np.abs(d[:rows].astype(np.float64) - exact) <= ulp).all()
    q, s, Wp = lora.merge_requant(W, A, B, scaling)
    gm = data[f"lora/{name}/merged"]
    # merged weights differ at most by 1 fp16 ulp from the reference's CPU pipeline
    diff = np.abs(Wp[:rows].astype(np.float32) - gm.astype(np.float32))
    assert (diff <= np.spacing(np.abs(gm)).astype(np.float32)).all()
    # requantisation of the reference's own merged weight is bit-exact
    assert gm.shape[0] == n
    q_ref, s_ref = quant.quantize_weight_int8(gm, F16)
    assert np.array_equal(q_ref, data[f"lora/{name}/q"])
    assert np.array_equal(s_ref, data[f"lora/{name}/scale"])
    assert sha(q_ref) == ent["q_sha256"]
    reg = lora.registry_delta(A, B, scaling)
    gr = data[f"lora/{name}/registry_delta"]
    assert np.abs(reg[:rows].astype(np.float32) - gr.astype(np.float32)).max() <= np.abs(gr).max() * 2e-3 + 1e-6


def test_add_delta_oracle():
    W = inputs.weight(11, 64, 128, F16, std=1.0)
    D = inputs.weight(12, 64, 128, F16, std=1.0)
    out = lora.add_delta(W, D)
    ref = (W.astype(np.float32) + D.astype(np.float32)).astype(np.float16)
    assert np.array_equal(out, ref)


def test_bf16_rounding_helper_matches_torch():
    torch = pytest.importorskip("torch")
    from oracle.numerics import f32_to_bf16_bits

    x = np.random.default_rng(0).standard_normal(100_000).astype(np.float32) * 3
    x[:3] = [np.inf, -np.inf, 0.0]
    t = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(f32_to_bf16_bits(x), t)
