"""GPU parity against the reference's own CUDA operators, compiled for sm_100a.

``oracle/build_ref.py`` compiles the reference extension's sources
(src/blackwell_ops/cuda/{basic_ops,kv_quant,lora_ops,lora_tiled}.cu) with the
reference loader's flags (``-O3 --use_fast_math``) into ``oracle/_ref``; these
tests run those kernels on the same inputs as this library's and the CPU
oracle, so the oracle itself is pinned to the reference's compiled kernels:

* ``lora_delta`` / ``lora_delta_tiled`` / ``add_delta_``: the CPU oracle's
  j-ordered fp32 restatement equals the reference kernels bit for bit; this
  library's tensor-core ΔW is within one fp16 ulp of them on < 1 % of values
  and ``add_delta_`` is bit-exact.
* ``quantize_kv_int8`` / ``dequantize_kv_int8``: the reference build's
  ``--use_fast_math`` replaces the two divisions with approximations, so its
  scales may differ from the IEEE quotient by up to 2 fp32 ulps and its codes
  by one step where a quotient lies that close to a half-way point; dequantising
  the same codes is bit-exact.
* ``fused_residual_rmsnorm`` / ``rmsnorm``: within one output ulp (the
  reference's fast-math reciprocal square root and contracted sums).
* SwiGLU: this library's fused gate/up GEMM against the reference ``swiglu``
  applied to two ``int8_gemm`` outputs: within two output ulps (each of g, u
  may round one ulp apart between the two plans; fast-math exp).

Skipped when the checker module is absent (built only where the reference
tree is present).
"""
import sys
from pathlib import Path

import numpy as np
import pytest

from oracle import kv, lora, norm
from oracle.numerics import F16

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

REF_DIR = Path(__file__).resolve().parent.parent / "oracle" / "_ref"


@pytest.fixture(scope="module")
def ref():
    if not list(REF_DIR.glob("bw_ref_ops*.so")):
        pytest.skip("reference checker module not built (oracle/build_ref.py)")
    sys.path.insert(0, str(REF_DIR))
    import bw_ref_ops

    return bw_ref_ops


def _rng(seed):
    return np.random.Generator(np.random.PCG64(seed))


def _h(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _ulp_diff(a, b):
    """|a - b| in units of fp16 ulp of b (arrays of float16)."""
    a = a.astype(np.float64)
    b64 = b.astype(np.float64)
    return np.abs(a - b64) / np.spacing(np.abs(b).astype(np.float16)).astype(np.float64)


@pytest.mark.parametrize("r,n,k", [(16, 256, 512), (128, 384, 1024), (64, 1000, 520), (7, 130, 200)])
def test_lora_delta_matches_reference_kernels(ref, cuda_dev, r, n, k):
    from blackwell_ops.cuda import lora_delta

    rng = _rng(r * n + k)
    A = (rng.standard_normal((r, k), dtype=np.float32) / np.sqrt(k)).astype(np.float16)
    B = (rng.standard_normal((n, r), dtype=np.float32) * 0.01).astype(np.float16)
    Ad, Bd = _h(A, cuda_dev), _h(B, cuda_dev)
    want = lora.lora_delta(A, B, 2.0)
    for fn in (ref.lora_delta, ref.lora_delta_tiled):
        got = fn(Ad, Bd, 2.0).cpu().numpy()
        assert np.array_equal(got.view(np.uint16), want.view(np.uint16)), f"oracle != reference {fn.__name__}"
    ours = lora_delta(Ad, Bd, 2.0).cpu().numpy()
    d = _ulp_diff(ours, want)
    assert d.max() <= 1.0 and (d > 0).mean() < 0.01


def test_add_delta_matches_reference_kernel(ref, cuda_dev):
    from blackwell_ops.cuda import add_delta_

    rng = _rng(5)
    W = (rng.standard_normal((300, 700), dtype=np.float32) * 0.02).astype(np.float16)
    D = (rng.standard_normal((300, 700), dtype=np.float32) * 0.003).astype(np.float16)
    a, b = _h(W, cuda_dev), _h(W, cuda_dev)
    ref.add_delta_(a, _h(D, cuda_dev))
    add_delta_(b, _h(D, cuda_dev))
    assert torch.equal(a, b)
    assert np.array_equal(a.cpu().numpy().view(np.uint16), lora.add_delta(W, D).view(np.uint16))


@pytest.mark.parametrize("c,n", [(32, 4096), (64, 8192), (128, 16384), (5, 1000)])
def test_kv_quant_against_reference_build(ref, cuda_dev, c, n):
    from blackwell_ops.cuda import dequantize_kv_int8, quantize_kv_int8

    x = _rng(c + n).standard_normal((c, n), dtype=np.float32).astype(np.float16)
    xd = _h(x, cuda_dev)
    q_ref, s_ref = ref.quantize_kv_int8(xd)
    q, s = quantize_kv_int8(xd)
    s_ref_n, s_n = s_ref.cpu().numpy(), s.cpu().numpy()
    ulps = np.abs(s_ref_n.view(np.int32).astype(np.int64) - s_n.view(np.int32).astype(np.int64))
    assert ulps.max() <= 2, f"scale differs by {ulps.max()} fp32 ulps"
    dq = np.abs(q_ref.cpu().numpy().astype(np.int32) - q.cpu().numpy().astype(np.int32))
    assert dq.max() <= 1 and (dq > 0).mean() < 1e-3
    # our codes are the IEEE ones
    qo, so = kv.quantize_kv_int8(x)
    assert np.array_equal(q.cpu().numpy(), qo) and np.array_equal(s_n.view(np.uint32), so.view(np.uint32))
    # dequantisation of the same codes and scales: bit-exact with the reference kernel
    assert torch.equal(ref.dequantize_kv_int8(q, s).view(torch.int16), dequantize_kv_int8(q, s).view(torch.int16))


@pytest.mark.parametrize("m,k", [(64, 512), (16, 4096), (3, 28672)])
def test_rmsnorm_against_reference_build(ref, cuda_dev, m, k):
    from blackwell_ops.cuda import fused_residual_rmsnorm, rmsnorm

    rng = _rng(m * k)
    x, r, w = (rng.standard_normal(s, dtype=np.float32).astype(np.float16) for s in ((m, k), (m, k), (k,)))
    xd, rd, wd = _h(x, cuda_dev), _h(r, cuda_dev), _h(w, cuda_dev)
    for got, want in ((fused_residual_rmsnorm(xd, rd, wd), ref.fused_residual_rmsnorm(xd, rd, wd, 1e-6)),
                      (rmsnorm(xd, wd), ref.rmsnorm(xd, wd, 1e-6))):
        d = _ulp_diff(got.cpu().numpy(), want.cpu().numpy())
        assert d.max() <= 1.0, d.max()
    # and our kernel is the restatement, bit for bit
    out = fused_residual_rmsnorm(xd, rd, wd).cpu().numpy()
    assert np.array_equal(out.view(np.uint16), norm.residual_rmsnorm(x, r, w, 1e-6, F16).view(np.uint16))


def test_swiglu_gemm_against_reference_swiglu(ref, cuda_dev):
    from blackwell_ops.kernels import int8_gemm, int8_gemm_swiglu, quantize_weight_int8

    g = torch.Generator(device=cuda_dev).manual_seed(3)
    x = torch.randn(16, 1024, generator=g, device=cuda_dev).half()
    wg, sg = quantize_weight_int8((torch.randn(3072, 1024, generator=g, device=cuda_dev) * 0.02).half())
    wu, su = quantize_weight_int8((torch.randn(3072, 1024, generator=g, device=cuda_dev) * 0.02).half())
    fused = int8_gemm_swiglu(x, wg, sg, wu, su)
    want = ref.swiglu(int8_gemm(x, wg, sg), int8_gemm(x, wu, su))
    d = _ulp_diff(fused.cpu().numpy(), want.cpu().numpy())
    # g and u may each differ by one ulp between the fused plan and two separate GEMMs (fp32 sums in
    # another order), and the reference's fast-math exp by a few fp32 ulps: at most 2 output ulps
    assert d.max() <= 2.0, d.max()
    assert (d > 1.0).mean() < 1e-3
