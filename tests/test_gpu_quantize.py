"""GPU parity: bw_quantize_rowwise_int8 vs the reference's bits (golden fixtures + oracle)."""
import hashlib

import numpy as np
import pytest

from cases import EDGE_CASES, QUANT_CASES, edge_weight
from oracle import inputs, quant
from oracle.numerics import BF16, F16, F32

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def to_dev(a, dt, dev):
    if dt == BF16:
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(dev)
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def to_np(t, dt):
    t = t.cpu().contiguous()
    if dt == BF16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def ops():
    from blackwell_ops import _lib
    from blackwell_ops.kernels import quantize_weight_int8

    yield quantize_weight_int8
    assert _lib.device_status() == 0


@pytest.mark.parametrize("case", QUANT_CASES, ids=[c[0] for c in QUANT_CASES])
def test_quantize_bit_exact_vs_reference(case, golden, cuda_dev, ops):
    name, seed, n, k, dt = case
    _, index = golden
    w = to_dev(inputs.weight(seed, n, k, dt), dt, cuda_dev)
    q, s = ops(w)
    torch.cuda.synchronize()
    assert sha(q.cpu().numpy()) == index["quant"][name]["q_sha256"]
    assert sha(to_np(s, dt)) == index["quant"][name]["scale_sha256"]


@pytest.mark.parametrize("case", EDGE_CASES, ids=[c[0] for c in EDGE_CASES])
def test_quantize_edge_rows(case, golden, cuda_dev, ops):
    name, dt = case
    data, _ = golden
    w = edge_weight(name, dt)
    q, s = ops(to_dev(w, dt, cuda_dev))
    assert np.array_equal(q.cpu().numpy(), data[f"edge/{name}/q"])
    want = np.ascontiguousarray(data[f"edge/{name}/scale"])
    got = np.ascontiguousarray(to_np(s, dt))
    assert got.dtype == want.dtype and got.tobytes() == want.tobytes()  # bitwise: NaN scales included


@pytest.mark.parametrize("dt", [F16, BF16, F32])
def test_quantize_strided_and_batched(dt, cuda_dev, ops):
    base = inputs.weight(77, 64, 1000, dt)
    wd = to_dev(base, dt, cuda_dev)
    for off in (8, 3):  # row stride 1000: 16-byte aligned rows (vector path) and unaligned (two-pass path)
        q, s = ops(wd[:, off:off + 512])
        qo, so = quant.quantize_weight_int8(base[:, off:off + 512], dt)
        assert np.array_equal(q.cpu().numpy(), qo)
        assert np.array_equal(to_np(s, dt), so)
    # leading dims are flattened exactly like amax(dim=-1)
    w3 = wd[:48, :512].reshape(3, 16, 512)
    q3, s3 = ops(w3)
    assert q3.shape == (3, 16, 512) and s3.shape == (3, 16)
    q2, s2 = ops(wd[:48, :512].contiguous())
    assert torch.equal(q3.reshape(48, 512), q2) and torch.equal(s3.reshape(48), s2)


@pytest.mark.parametrize("k", [1, 7, 8, 9, 255, 4096 + 3, 16384, 32768, 40000])
def test_quantize_row_lengths(k, cuda_dev, ops):
    """Register-resident path for every group width, ragged tails and the two-pass path."""
    w = inputs.weight(500 + k, 33, k, F16, std=0.5)
    q, s = ops(to_dev(w, F16, cuda_dev))
    qo, so = quant.quantize_weight_int8(w, F16)
    assert np.array_equal(q.cpu().numpy(), qo)
    assert np.array_equal(s.cpu().numpy(), so)


def test_quantize_full_size_70b_properties(cuda_dev, ops):
    """Full Llama-3-70B MLP shard size: sampled rows bit-exact, and size-independent properties."""
    n, k = 28672, 8192
    g = torch.Generator(device=cuda_dev).manual_seed(5)
    w = (torch.randn(n, k, generator=g, device=cuda_dev) * 0.02).to(torch.bfloat16)
    q, s = ops(w)
    rows = torch.randint(0, n, (64,), generator=g, device=cuda_dev)
    wr = w[rows].cpu().view(torch.int16).numpy().view(np.uint16)
    qo, so = quant.quantize_weight_int8(wr, BF16)
    assert np.array_equal(q[rows].cpu().numpy(), qo)
    assert np.array_equal(s[rows].cpu().view(torch.int16).numpy().view(np.uint16), so)
    assert int(q.abs().max()) == 127
    # every row reaches +-127 at its absmax element (up to the scale's rounding)
    assert int((q.abs().amax(dim=1) >= 126).sum()) == n
    # |q*s - w| <= 0.75 s: half a code from rint plus up to a quarter code from
    # rounding the quotient to bf16 (spacing 0.5 between 64 and 128)
    err = (q.float() * s.float()[:, None] - w.float()).abs()
    assert bool((err <= s.float()[:, None] * 0.75 * 1.01 + 1e-12).all())


def test_quantize_empty_and_errors(cuda_dev, ops):
    q, s = ops(torch.empty(0, 16, dtype=torch.float16, device=cuda_dev))
    assert q.shape == (0, 16) and s.shape == (0,)
    with pytest.raises(RuntimeError):
        ops(torch.empty(4, 0, dtype=torch.float16, device=cuda_dev))
    with pytest.raises(RuntimeError):
        ops(torch.ones(4, 4, dtype=torch.int32, device=cuda_dev))
    with pytest.raises(RuntimeError):
        ops(torch.ones(4, 4, dtype=torch.float16))
