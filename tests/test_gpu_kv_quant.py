"""GPU parity: the KV-cache quantiser (bw_quantize_kv_int8 / bw_dequantize_kv_int8).

Bit-exact against the CPU restatement of the reference's kernels
(oracle/kv.py, src/blackwell_ops/cuda/kv_quant.cu:17-58): codes, fp32 scales
and dequantised fp16 values, over channel lengths that take every launch path
(one to eight CTAs per channel, 1..4 chunks per thread, the two-pass kernel
for long or unaligned rows, strided rows) and rows holding NaN, inf, zeros and
exact half-way quotients.  Also the reference test's own round trip
(src/blackwell_ops/tests/test_kv_quant.py: C=32, N=4096, max error < 0.1).
"""
import numpy as np
import pytest

from oracle import kv

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _rows(seed, c, n):
    rng = np.random.Generator(np.random.PCG64(seed))
    return rng.standard_normal((c, n), dtype=np.float32).astype(np.float16)


def _check(x_np, dev, x_dev=None):
    from blackwell_ops.cuda import dequantize_kv_int8, quantize_kv_int8

    xd = torch.from_numpy(x_np).to(dev) if x_dev is None else x_dev
    q, s = quantize_kv_int8(xd)
    qo, so = kv.quantize_kv_int8(x_np)
    assert q.dtype == torch.int8 and s.dtype == torch.float32
    assert np.array_equal(s.cpu().numpy().view(np.uint32), so.view(np.uint32)), "scales differ"
    qn = q.cpu().numpy()
    bad = np.argwhere(qn != qo)
    assert bad.size == 0, f"{len(bad)} codes differ, first at {bad[:4].tolist()}"
    xr = dequantize_kv_int8(q, s)
    assert xr.dtype == torch.float16
    want = kv.dequantize_kv_int8(qo, so)
    assert np.array_equal(xr.cpu().numpy().view(np.uint16), want.view(np.uint16)), "dequantised values differ"


@pytest.mark.parametrize("c,n", [(1, 8), (3, 1), (2, 7), (32, 4096), (64, 8192), (128, 16384), (5, 2048 + 8),
                                 (4, 8 * 8192), (3, 8 * 8192 + 8), (2, 100003), (7, 24576)])
def test_kv_quant_bit_exact(cuda_dev, c, n):
    _check(_rows(c * 1000 + n, c, n), cuda_dev)


def test_kv_quant_strided_rows(cuda_dev):
    x = _rows(11, 16, 4104)
    xd = torch.from_numpy(x).to(cuda_dev)[:, 8:4104 - 8]  # row stride 4104, 16-byte aligned start
    _check(np.ascontiguousarray(x[:, 8:4104 - 8]), cuda_dev, xd)
    xu = torch.from_numpy(x).to(cuda_dev)[:, 3:4003]  # unaligned start: the two-pass kernel
    _check(np.ascontiguousarray(x[:, 3:4003]), cuda_dev, xu)


def test_kv_quant_edge_rows(cuda_dev):
    n = 4096
    x = _rows(5, 8, n)
    x[0] = 0.0                          # all zeros: scale 0, codes 0
    x[1, ::3] = np.nan                  # NaN ignored by the max, coded 0
    x[2, 17] = np.inf                   # inf scale: every code 0
    x[3] = np.float16(0.0)
    x[3, 1] = np.float16(127.0)         # scale 1: exact half-way quotients round to even
    x[3, 2:10] = np.array([0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 126.5, -126.5], dtype=np.float16)
    x[4] = np.nan                       # all NaN
    x[5, :] = np.float16(6.0e-8)        # fp16 subnormals
    x[6, 5] = np.float16(-65504.0)      # largest magnitude
    _check(x, cuda_dev)


def test_kv_quant_reference_roundtrip(cuda_dev):
    from blackwell_ops.cuda import dequantize_kv_int8, quantize_kv_int8

    torch.manual_seed(0)
    x = torch.randn(32, 4096, device=cuda_dev, dtype=torch.float16)
    q, scale = quantize_kv_int8(x)
    err = (x.float() - dequantize_kv_int8(q, scale).float()).abs().max().item()
    assert err < 0.1
    assert q.dtype == torch.int8 and scale.dtype == torch.float32


def test_kv_quant_errors(cuda_dev):
    from blackwell_ops.cuda import dequantize_kv_int8, quantize_kv_int8

    with pytest.raises(RuntimeError, match="x must be CUDA fp16"):
        quantize_kv_int8(torch.zeros(2, 8, device=cuda_dev, dtype=torch.float32))
    with pytest.raises(RuntimeError, match=r"x must be \[C, N\]"):
        quantize_kv_int8(torch.zeros(8, device=cuda_dev, dtype=torch.float16))
    with pytest.raises(RuntimeError, match="scale must be CUDA fp32"):
        dequantize_kv_int8(torch.zeros(2, 8, device=cuda_dev, dtype=torch.int8),
                           torch.zeros(2, device=cuda_dev, dtype=torch.float16))
