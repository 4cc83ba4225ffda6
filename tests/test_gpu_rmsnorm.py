"""GPU parity: residual + RMSNorm, alone and as the W8A16 GEMM's prologue.

* fused_residual_rmsnorm / rmsnorm (bw_residual_rmsnorm) bit for bit against the CPU
  restatement of the reference kernels in their summation order (oracle/norm.py,
  src/blackwell_ops/cuda/basic_ops.cu:16-78), fp16 and bf16, row lengths 1 .. 28672;
* the reference test's own check (test_cuda_basic.py:21-30, tolerance 0.01);
* int8_gemm_rmsnorm (bw_w8a16_gemm_rmsnorm): bit-identical to fused_residual_rmsnorm followed
  by int8_gemm, and within the GEMM tolerance of the fp32 dequantise-then-matmul of the oracle's
  normalised rows.
"""
import numpy as np
import pytest

from oracle import gemm, norm, quant
from oracle.numerics import BF16, F16, from_f32, to_f32

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _dev(a, dt, dev):
    if dt == BF16:
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(dev)
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _np(t, dt):
    if dt == BF16:
        return t.view(torch.int16).cpu().numpy().view(np.uint16)
    return t.cpu().numpy()


def _case(seed, m, k, dt):
    rng = np.random.Generator(np.random.PCG64(seed))
    mk = lambda shape: from_f32(rng.standard_normal(shape, dtype=np.float32), dt)  # noqa: E731
    return mk((m, k)), mk((m, k)), mk((k,))


@pytest.mark.parametrize("dt", [F16, BF16])
@pytest.mark.parametrize("m,k", [(1, 1), (3, 255), (64, 512), (16, 4096), (16, 8192), (2, 28672), (5, 1000)])
def test_residual_rmsnorm_bit_exact(cuda_dev, dt, m, k):
    from blackwell_ops.cuda import fused_residual_rmsnorm, rmsnorm

    x, r, w = _case(m * 31 + k, m, k, dt)
    out = fused_residual_rmsnorm(_dev(x, dt, cuda_dev), _dev(r, dt, cuda_dev), _dev(w, dt, cuda_dev))
    want = norm.residual_rmsnorm(x, r, w, 1e-6, dt)
    assert np.array_equal(_np(out, dt).view(np.uint16), np.asarray(want).view(np.uint16))
    out = rmsnorm(_dev(x, dt, cuda_dev), _dev(w, dt, cuda_dev), eps=1e-5)
    want = norm.residual_rmsnorm(x, None, w, 1e-5, dt)
    assert np.array_equal(_np(out, dt).view(np.uint16), np.asarray(want).view(np.uint16))


def test_reference_test_tolerance(cuda_dev):
    from blackwell_ops.cuda import fused_residual_rmsnorm

    torch.manual_seed(0)
    M, N = 64, 512
    x = torch.randn(M, N, device=cuda_dev, dtype=torch.float16)
    r = torch.randn(M, N, device=cuda_dev, dtype=torch.float16)
    w = torch.randn(N, device=cuda_dev, dtype=torch.float16)
    out = fused_residual_rmsnorm(x, r, w)
    x_f = (x + r).float()
    ref = x_f / torch.sqrt((x_f * x_f).mean(dim=-1, keepdim=True) + 1e-6) * w.float()
    assert (out.float() - ref).abs().max().item() < 0.01


@pytest.mark.parametrize("dt", [F16, BF16])
@pytest.mark.parametrize("m,n,k,with_res", [(16, 3072, 1024, True), (1, 1024, 4096, False), (64, 2048, 2048, True),
                                           (16, 8192, 28672, True), (5, 300, 1000, True)])
def test_int8_gemm_rmsnorm(cuda_dev, dt, m, n, k, with_res):
    from blackwell_ops.cuda import fused_residual_rmsnorm, rmsnorm
    from blackwell_ops.kernels import int8_gemm, int8_gemm_rmsnorm

    x, r, nw = _case(7 * m + n + k, m, k, dt)
    rng = np.random.Generator(np.random.PCG64(n))
    wt = from_f32(rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02), dt)
    q, s = quant.quantize_weight_int8(wt, dt)
    xd, rd, nwd = _dev(x, dt, cuda_dev), _dev(r, dt, cuda_dev), _dev(nw, dt, cuda_dev)
    qd, sd = torch.from_numpy(q).to(cuda_dev), _dev(s, dt, cuda_dev)
    y = int8_gemm_rmsnorm(xd, rd if with_res else None, nwd, qd, sd)
    xn = fused_residual_rmsnorm(xd, rd, nwd) if with_res else rmsnorm(xd, nwd)
    y2 = int8_gemm(xn, qd, sd)
    torch.cuda.synchronize()
    assert torch.equal(y.view(torch.int16), y2.view(torch.int16)), "fused prologue differs from the two ops"
    xn_o = norm.residual_rmsnorm(x, r if with_res else None, nw, 1e-6, dt)
    want = gemm.exact(xn_o, dt, q, s, dt)
    got = y.float().cpu().numpy().astype(np.float64)
    err = np.abs(got - want)
    if dt == F16:
        assert err.max() <= 1e-2
        assert np.linalg.norm(got - want) / np.linalg.norm(want) <= 1e-3
    else:
        assert (err <= 1e-2 + 2.0 ** -8 * np.abs(want)).all()
    from blackwell_ops import _lib

    assert _lib.device_status() == 0


@pytest.mark.parametrize("m,n,k", [(1, 3072, 1024), (16, 3072, 1024), (16, 1024, 4096)])
def test_prologue_leaves_shared_counters_zero(cuda_dev, m, n, k):
    """The normalised rows live in the caller's workspace, which int8_gemm shares: whatever the
    GEMM's plan (with or without split tiles), the counter region at its start stays zero."""
    from blackwell_ops import _lib
    from blackwell_ops.kernels import int8_gemm_rmsnorm
    from blackwell_ops.kernels.int8_gemm import _workspaces

    g = torch.Generator(device=cuda_dev).manual_seed(m + n + k)
    x = torch.randn(m, k, generator=g, device=cuda_dev).half()
    nw = torch.randn(k, generator=g, device=cuda_dev).half()
    q = torch.randint(-127, 128, (n, k), generator=g, device=cuda_dev, dtype=torch.int8)
    s = (torch.rand(n, generator=g, device=cuda_dev) * 1e-3 + 1e-4).half()
    int8_gemm_rmsnorm(x, None, nw, q, s)
    torch.cuda.synchronize()
    ws = _workspaces[(cuda_dev.index if cuda_dev.index is not None else torch.cuda.current_device(),
                      _lib.stream_ptr(cuda_dev))]
    assert int(ws[:4096].count_nonzero()) == 0
