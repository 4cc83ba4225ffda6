"""GPU parity of the fused gate/up W8A16 GEMM + SwiGLU (bw_w8a16_gemm_swiglu).

Reference composition: swiglu(int8_gemm(x, w_gate, s_gate), int8_gemm(x, w_up, s_up)),
the swiglu being the reference kernel's fp32 ``g / (1 + exp(-g)) * u`` rounded once
(src/blackwell_ops/cuda/basic_ops.cu:112-122).  Bound, elementwise: the kernel's g and u
are each within one output ulp (plus the fp32 accumulation error) of the exactly rounded
products, so |y - y_ref| <= 1.1 |u| e_g + |silu(g)| e_u + e_g e_u + ulp(y), with silu' <= 1.1.
"""
import numpy as np
import pytest

from oracle import gemm, inputs, quant
from oracle.numerics import BF16, F16, to_f32

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def to_dev(a, dt, dev):
    if dt == BF16:
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(dev)
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def spacing(v, dt):
    if dt == F16:
        return np.spacing(np.abs(v).astype(np.float16)).astype(np.float64)
    return np.maximum(np.abs(v), 2.0 ** -126) * 2.0 ** -7


def check_against_oracle(y, x, dt, qg, sg, qu, su):
    g = to_f32(gemm.int8_gemm(x, dt, qg, sg, dt), dt).astype(np.float64)
    u = to_f32(gemm.int8_gemm(x, dt, qu, su, dt), dt).astype(np.float64)
    want = to_f32(gemm.int8_gemm_swiglu(x, dt, qg, sg, qu, su, dt), dt).astype(np.float64)
    absx = np.abs(to_f32(x, dt).astype(np.float64))
    eg = spacing(g, dt) + 2.0 ** -22 * (absx @ np.abs(qg.astype(np.float64)).T) * np.abs(to_f32(sg, dt))[None, :]
    eu = spacing(u, dt) + 2.0 ** -22 * (absx @ np.abs(qu.astype(np.float64)).T) * np.abs(to_f32(su, dt))[None, :]
    silu = g / (1.0 + np.exp(-g))
    bound = 1.1 * np.abs(u) * eg + np.abs(silu) * eu + eg * eu + spacing(want, dt)
    got = y.float().cpu().numpy().astype(np.float64)
    assert np.all(np.abs(got - want) <= bound + 1e-30), float(np.max(np.abs(got - want) - bound))
    return float((got != want).mean())


@pytest.fixture(scope="module")
def op():
    from blackwell_ops import _lib
    from blackwell_ops.kernels import int8_gemm_swiglu

    yield int8_gemm_swiglu
    assert _lib.device_status() == 0


@pytest.mark.parametrize("m,n,k,dt", [(16, 3072, 1024, F16), (1, 1000, 512, F16), (4, 200, 4096, BF16),
                                      (64, 384, 1024, BF16), (130, 3072, 1024, F16), (300, 96, 256, BF16)])
def test_swiglu_vs_oracle(m, n, k, dt, cuda_dev, op):
    x = inputs.activations(m + 1, m, k, dt)
    qg, sg = quant.quantize_weight_int8(inputs.weight(n + 2, n, k, dt), dt)
    qu, su = quant.quantize_weight_int8(inputs.weight(n + 3, n, k, dt), dt)
    y = op(to_dev(x, dt, cuda_dev), torch.from_numpy(qg).to(cuda_dev), to_dev(sg, dt, cuda_dev),
           torch.from_numpy(qu).to(cuda_dev), to_dev(su, dt, cuda_dev))
    frac = check_against_oracle(y, x, dt, qg, sg, qu, su)
    assert frac < 0.02


def test_swiglu_cuda_core_path(cuda_dev, op):
    """Row strides TMA cannot address go to the CUDA-core kernel with the same arithmetic."""
    dt = F16
    x = inputs.activations(7, 16, 1027, dt)
    qg, sg = quant.quantize_weight_int8(inputs.weight(8, 130, 1024, dt), dt)
    qu, su = quant.quantize_weight_int8(inputs.weight(9, 130, 1024, dt), dt)
    xd = to_dev(x, dt, cuda_dev)[:, :1024]
    y = op(xd, torch.from_numpy(qg).to(cuda_dev), to_dev(sg, dt, cuda_dev), torch.from_numpy(qu).to(cuda_dev),
           to_dev(su, dt, cuda_dev))
    check_against_oracle(y, np.ascontiguousarray(x[:, :1024]), dt, qg, sg, qu, su)


@pytest.mark.parametrize("m,n,k", [(16, 14336, 4096), (2048, 14336, 4096), (16, 28672, 8192)])
def test_swiglu_full_size_vs_unfused(m, n, k, cuda_dev, op):
    """Llama-3-8B / 70B MLP sizes: the fused op against this library's own unfused composition
    (int8_gemm twice, then the reference swiglu arithmetic in torch fp32); bit-identical except
    where the two plans' fp32 summation orders round g or u differently."""
    from blackwell_ops.kernels import int8_gemm, quantize_weight_int8

    gen = torch.Generator(device=cuda_dev).manual_seed(m + n)
    qg, sg = quantize_weight_int8((torch.randn(n, k, generator=gen, device=cuda_dev) * 0.02).to(torch.bfloat16))
    qu, su = quantize_weight_int8((torch.randn(n, k, generator=gen, device=cuda_dev) * 0.02).to(torch.bfloat16))
    x = torch.randn(m, k, generator=gen, device=cuda_dev).to(torch.bfloat16)
    y = op(x, qg, sg, qu, su)
    g = int8_gemm(x, qg, sg).float()
    u = int8_gemm(x, qu, su).float()
    ref = (g / (1.0 + torch.exp(-g)) * u).to(torch.bfloat16)
    diff = (y.double() - ref.double()).abs()
    ulp = torch.clamp(ref.double().abs(), min=2.0 ** -126) * 2.0 ** -7
    bound = 1.1 * u.double().abs() * 2.0 ** -7 * g.double().abs() + g.double().abs() * 2.0 ** -7 * u.double().abs()
    assert bool((diff <= bound + 2 * ulp + 1e-6).all()), float((diff - bound - 2 * ulp).max())
    assert float((y != ref).float().mean()) < 0.02


def test_swiglu_errors(cuda_dev, op):
    x = torch.randn(4, 64, device=cuda_dev, dtype=torch.float16)
    q = torch.zeros(8, 64, device=cuda_dev, dtype=torch.int8)
    s = torch.ones(8, device=cuda_dev, dtype=torch.float16)
    with pytest.raises(RuntimeError):
        op(x, q, s, q[:4], s)
    with pytest.raises(RuntimeError):
        op(x, q, s, q, s.float())
    with pytest.raises(RuntimeError):
        op(x.cpu(), q, s, q, s)
    assert op(x[:0], q, s, q, s).shape == (0, 8)
