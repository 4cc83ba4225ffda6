"""GPU parity: the tcgen05 W8A16 GEMM (bw_w8a16_gemm) vs the oracle.

Tolerance: against the fp32-accumulated
dequantise-then-matmul, fp16 outputs must have max |err| <= 1e-2 and relative
(Frobenius) error <= 1e-3.  bf16 outputs carry 8 significant bits, so their
bound is |err| <= 1e-2 + 2^-8 |ref| elementwise (one bf16 ulp).  In addition
every output must be within one output ulp of dt(fp32(exact acc) * scale),
the value the reference kernel rounds (int8_gemm.py:52-58).
"""
import ctypes

import numpy as np
import pytest

from cases import GEMM_CASES
from oracle import gemm, inputs, quant
from oracle.numerics import BF16, F16, F32, to_f32

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

TDT = {F16: "float16", BF16: "bfloat16", F32: "float32"}


def to_dev(a, dt, dev):
    if dt == BF16:
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(dev)
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def check_tol(y, ref64, dt):
    yv = y.float().cpu().numpy().astype(np.float64)
    err = np.abs(yv - ref64)
    if dt == F16:
        assert err.max() <= 1e-2, err.max()
        rel = np.linalg.norm(yv - ref64) / max(np.linalg.norm(ref64), 1e-30)
        assert rel <= 1e-3, rel
    else:
        assert (err <= 1e-2 + 2.0 ** -8 * np.abs(ref64)).all(), err.max()


def check_ulp(y, x, xdt, q, s, sdt):
    """Within one output ulp of the reference kernel's own rounding of the exact
    accumulator, plus the fp32 accumulation error any summation order carries
    (bounded here by 2^-22 * sum_k |x q| * |scale|, which matters only for
    outputs near zero)."""
    want = to_f32(gemm.int8_gemm(x, xdt, q, s, sdt), xdt).astype(np.float64)
    got = y.float().cpu().numpy().astype(np.float64)
    if xdt == F16:
        ulp = np.spacing(np.abs(want).astype(np.float16)).astype(np.float64)
    else:
        ulp = np.maximum(np.abs(want), 2.0 ** -126) * 2.0 ** -7
    absacc = np.abs(to_f32(x, xdt).astype(np.float64)) @ np.abs(q.astype(np.float64)).T
    acc_err = 2.0 ** -22 * absacc * np.abs(to_f32(s, sdt).astype(np.float64))[None, :]
    assert (np.abs(got - want) <= ulp + acc_err + 1e-30).all()
    return float((got != want).mean())


@pytest.fixture(scope="module")
def ops():
    from blackwell_ops import _lib
    from blackwell_ops.kernels import int8_gemm

    yield int8_gemm
    assert _lib.device_status() == 0


def run_case(ops, dev, m, n, k, xdt=F16, sdt=F16, seed=0, x_pad=0):
    wdt = sdt if sdt != F32 else F32
    w = inputs.weight(seed, n, k, wdt)
    q, s = quant.quantize_weight_int8(w, wdt)
    x = inputs.activations(seed + 1, m, k + x_pad, xdt)
    xd = to_dev(x, xdt, dev)[:, :k]
    xo = x[:, :k]
    y = ops(xd, torch.from_numpy(q).to(dev), to_dev(s, sdt, dev))
    assert y.dtype == getattr(torch, TDT[xdt]) and tuple(y.shape) == (m, n)
    check_tol(y, gemm.exact(xo, xdt, q, s, sdt), xdt)
    return check_ulp(y, xo, xdt, q, s, sdt)


@pytest.mark.parametrize("case", GEMM_CASES, ids=[c[0] for c in GEMM_CASES])
def test_gemm_golden_cases(case, golden, cuda_dev, ops):
    name, seed, m, n, k, xdt, wdt = case
    data, _ = golden
    x = inputs.activations(seed + 1, m, k, xdt)
    w = inputs.weight(seed, n, k, wdt)
    q, s = quant.quantize_weight_int8(w, wdt)
    y = ops(to_dev(x, xdt, cuda_dev), torch.from_numpy(q).to(cuda_dev), to_dev(s, wdt, cuda_dev))
    ref = data[f"gemm/{name}/ref_fp32"].astype(np.float64)  # the reference test's own expression
    check_tol(y, ref, xdt)
    check_ulp(y, x, xdt, q, s, wdt)


@pytest.mark.parametrize("m", [1, 2, 3, 4, 8, 15, 16, 17, 31, 32, 33, 63, 64, 65, 127, 128, 129, 300])
def test_gemm_token_counts(m, cuda_dev, ops):
    frac = run_case(ops, cuda_dev, m, 3072, 1024, seed=m)
    assert frac < 0.02


@pytest.mark.parametrize("n,k", [(96, 128), (40, 48), (200, 136), (1024, 3072), (2048, 1024), (130, 4096),
                                 (256, 120), (64, 100)])
@pytest.mark.parametrize("m", [1, 16, 64, 200])
def test_gemm_shapes(n, k, m, cuda_dev, ops):
    run_case(ops, cuda_dev, m, n, k, seed=n + k + m)


@pytest.mark.parametrize("xdt,sdt", [(F16, BF16), (F16, F32), (BF16, BF16), (BF16, F32), (BF16, F16)])
@pytest.mark.parametrize("m", [4, 48, 256])
def test_gemm_dtypes(xdt, sdt, m, cuda_dev, ops):
    run_case(ops, cuda_dev, m, 1024, 1024, xdt=xdt, sdt=sdt, seed=m + 7)


@pytest.mark.parametrize("m", [1, 16, 96])
def test_gemm_strided_x(m, cuda_dev, ops):
    run_case(ops, cuda_dev, m, 512, 1024, seed=99, x_pad=64)   # row stride 1088 (TMA path)
    run_case(ops, cuda_dev, m, 512, 1024, seed=98, x_pad=3)    # row stride 1027 (CUDA-core path)


def test_gemm_lm_head_shape(cuda_dev, ops):
    run_case(ops, cuda_dev, 16, 151936, 1024, seed=3)


def test_gemm_deterministic_and_reusable(cuda_dev, ops):
    """Split-K reduction is order-fixed and leaves its tile counters zeroed."""
    w = inputs.weight(1, 3072, 1024, F16)
    q, s = quant.quantize_weight_int8(w, F16)
    qd, sd = torch.from_numpy(q).to(cuda_dev), torch.from_numpy(s).to(cuda_dev)
    x = to_dev(inputs.activations(2, 16, 1024, F16), F16, cuda_dev)
    ys = [ops(x, qd, sd) for _ in range(5)]
    for y in ys[1:]:
        assert torch.equal(y, ys[0])


@pytest.mark.parametrize("m,n,k", [(16, 8192, 28672), (1, 1024, 28672), (64, 3072, 8192), (16, 28672, 8192),
                                   (130, 2048, 8192)])
def test_gemm_stream_k_cut_tiles(m, n, k, cuda_dev):
    """Shapes whose tiles are cut between several CTAs' k-ranges (stream-K): parity,
    bit-identical repeats through the C ABI with one workspace, counters back to zero."""
    from blackwell_ops import _lib

    lib = _lib.lib
    g = torch.Generator(device=cuda_dev).manual_seed(m + n + k)
    w = (torch.randn(n, k, generator=g, device=cuda_dev) * 0.02).to(torch.bfloat16)
    from blackwell_ops.kernels import quantize_weight_int8

    q, s = quantize_weight_int8(w)
    x = torch.randn(m, k, generator=g, device=cuda_dev).to(torch.bfloat16)
    need = lib.bw_w8a16_gemm_workspace_size(m, n, k)
    ws = torch.zeros(max(need, 16), dtype=torch.uint8, device=cuda_dev)
    st = _lib.stream_ptr(cuda_dev)
    ys = []
    for _ in range(3):
        y = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=cuda_dev)
        rc = lib.bw_w8a16_gemm(x.data_ptr(), 1, k, q.data_ptr(), k, s.data_ptr(), 1, y.data_ptr(), n, m, n, k,
                               ws.data_ptr(), ws.numel(), st)
        assert rc == 0, lib.bw_last_error()
        ys.append(y)
    torch.cuda.synchronize()
    ref = x.double() @ (q.double() * s.double()[:, None]).t()
    err = (ys[0].double() - ref).abs()
    assert bool((err <= 1e-2 + 2.0 ** -8 * ref.abs()).all()), float(err.max())
    assert all(torch.equal(y, ys[0]) for y in ys[1:])
    zeroed = lib.bw_w8a16_gemm_workspace_zeroed_bytes(m, n, k)
    assert int(ws[:zeroed].sum()) == 0
    assert _lib.device_status() == 0


def test_gemm_workspace_shared_across_shapes(cuda_dev):
    """One workspace serves a sequence of shapes with different plans (split-K, stream-K,
    cut tiles): each call's pieces never land on another shape's counters."""
    from blackwell_ops import _lib

    lib = _lib.lib
    shapes = [(16, 3072, 1024), (16, 151936, 1024), (1, 1024, 28672), (16, 3072, 1024), (64, 3072, 8192),
              (16, 151936, 1024)]
    need = max(lib.bw_w8a16_gemm_workspace_size(*sh) for sh in shapes)
    ws = torch.zeros(need, dtype=torch.uint8, device=cuda_dev)
    st = _lib.stream_ptr(cuda_dev)
    g = torch.Generator(device=cuda_dev).manual_seed(11)
    for m, n, k in shapes:
        q = torch.randint(-127, 128, (n, k), generator=g, device=cuda_dev, dtype=torch.int8)
        # scales keep |y| in the range where the absolute fp16 bound is meaningful (|y| < 8)
        s = ((torch.rand(n, generator=g, device=cuda_dev) * 1e-3 + 1e-4) * (1024.0 / k) ** 0.5).half()
        x = torch.randn(m, k, generator=g, device=cuda_dev).half()
        y = torch.full((m, n), float("nan"), dtype=torch.float16, device=cuda_dev)
        rc = lib.bw_w8a16_gemm(x.data_ptr(), 0, k, q.data_ptr(), k, s.data_ptr(), 0, y.data_ptr(), n, m, n, k,
                               ws.data_ptr(), ws.numel(), st)
        assert rc == 0, lib.bw_last_error()
        ref = x.double() @ (q.double() * s.double()[:, None]).t()
        err = (y.double() - ref).abs()
        assert float(err.max()) <= 1e-2 and float(err.norm() / ref.norm()) <= 1e-3, (m, n, k)
    assert int(ws[: lib.bw_w8a16_gemm_workspace_zeroed_bytes(16, 151936, 1024)].sum()) == 0
    assert _lib.device_status() == 0


@pytest.mark.parametrize("m,n,k", [(2048, 14336, 4096), (512, 4096, 14336), (4096, 8192, 2048), (8192, 14336, 4096),
                                   (8192, 4096, 14336)])
def test_gemm_prefill_full_size_vs_torch_fp32(m, n, k, cuda_dev, ops):
    """Full prefill sizes (cfg4's Llama-3-8B MLP shapes up to M = 8192): compared with the
    dequantise-matmul in fp64 on the GPU."""
    g = torch.Generator(device=cuda_dev).manual_seed(m + n)
    w = (torch.randn(n, k, generator=g, device=cuda_dev) * 0.02).to(torch.bfloat16)
    from blackwell_ops.kernels import quantize_weight_int8

    q, s = quantize_weight_int8(w)
    x = torch.randn(m, k, generator=g, device=cuda_dev).to(torch.bfloat16)
    y = ops(x, q, s)
    torch.backends.cuda.matmul.allow_tf32 = False
    ref = (x.double() @ (q.double() * s.double()[:, None]).t())
    err = (y.double() - ref).abs()
    assert bool((err <= 1e-2 + 2.0 ** -8 * ref.abs()).all()), float(err.max())


def test_gemm_errors(cuda_dev, ops):
    x = torch.randn(4, 64, device=cuda_dev, dtype=torch.float16)
    q = torch.zeros(8, 64, device=cuda_dev, dtype=torch.int8)
    s = torch.ones(8, device=cuda_dev, dtype=torch.float16)
    with pytest.raises(RuntimeError):
        ops(x.float(), q, s)
    with pytest.raises(RuntimeError):
        ops(x, q[:, :32], s)
    with pytest.raises(RuntimeError):
        ops(x.cpu(), q, s)
    assert ops(x[:0], q, s).shape == (0, 8)


def test_gemm_capi_workspace_contract(cuda_dev):
    """Through the C ABI: a split-K plan without workspace is refused with BW_ERR_WORKSPACE."""
    from blackwell_ops import _lib

    lib = _lib.lib
    m, n, k = 16, 1024, 4096
    need = lib.bw_w8a16_gemm_workspace_size(m, n, k)
    assert need > 0 and lib.bw_w8a16_gemm_workspace_zeroed_bytes(m, n, k) > 0
    x = torch.randn(m, k, device=cuda_dev, dtype=torch.float16)
    q = torch.ones(n, k, device=cuda_dev, dtype=torch.int8)
    s = torch.ones(n, device=cuda_dev, dtype=torch.float16)
    y = torch.empty(m, n, device=cuda_dev, dtype=torch.float16)
    st = _lib.stream_ptr(cuda_dev)
    rc = lib.bw_w8a16_gemm(x.data_ptr(), 0, k, q.data_ptr(), k, s.data_ptr(), 0, y.data_ptr(), n, m, n, k, None, 0, st)
    assert rc == _lib.BW_ERR_WORKSPACE
    assert b"workspace" in lib.bw_last_error()
    ws = torch.zeros(need, dtype=torch.uint8, device=cuda_dev)
    rc = lib.bw_w8a16_gemm(x.data_ptr(), 0, k, q.data_ptr(), k, s.data_ptr(), 0, y.data_ptr(), n, m, n, k,
                           ws.data_ptr(), need, st)
    assert rc == 0
    ref = x.float().sum(dim=1, keepdim=True).expand(m, n)
    assert torch.allclose(y.float(), ref, atol=1e-2, rtol=1e-3)
    assert int(ws[: lib.bw_w8a16_gemm_workspace_zeroed_bytes(m, n, k)].sum()) == 0
