"""CPU checks of the KV-cache quantiser oracle (oracle/kv.py) on hand-computed rows.

The reference's kernels (src/blackwell_ops/cuda/kv_quant.cu:17-58) run only on
a GPU, so these cases spell out the source's fp32 arithmetic by hand: the
channel maximum ignores NaN, scale = amax / 127 in fp32, codes round half to
even, NaN quotients become 0, dequantisation is one fp32 product rounded to
fp16.
"""
import numpy as np

from oracle import kv


def f16(*v):
    return np.array(v, dtype=np.float16)


def test_scale_and_codes_of_a_plain_row():
    x = f16(1.0, -2.0, 127.0, 0.5).reshape(1, -1)
    q, s = kv.quantize_kv_int8(x)
    assert s.dtype == np.float32 and s[0] == np.float32(127.0) / np.float32(127.0)
    assert q.tolist() == [[1, -2, 127, 0]]  # 0.5 / 1 rounds half to even -> 0


def test_half_way_quotients_round_to_even():
    x = f16(2.5, 3.5, -2.5, 127.0).reshape(1, -1)
    q, s = kv.quantize_kv_int8(x)
    assert s[0] == np.float32(1.0)
    assert q.tolist() == [[2, 4, -2, 127]]


def test_nan_is_ignored_by_the_max_and_coded_as_zero():
    x = f16(np.nan, 2.0, -4.0, 1.0).reshape(1, -1)
    q, s = kv.quantize_kv_int8(x)
    assert s[0] == np.float32(4.0) / np.float32(127.0)
    assert q[0, 0] == 0 and q[0, 2] == -127


def test_zero_and_all_nan_rows():
    x = np.stack([f16(0.0, -0.0, 0.0), f16(np.nan, np.nan, np.nan)])
    q, s = kv.quantize_kv_int8(x)
    assert s.tolist() == [0.0, 0.0]
    assert (q == 0).all()


def test_inf_channel_gives_inf_scale_and_zero_codes():
    x = f16(np.inf, 1.0, -3.0).reshape(1, -1)
    q, s = kv.quantize_kv_int8(x)
    assert np.isinf(s[0])
    assert q.tolist() == [[0, 0, 0]]


def test_dequantise_rounds_the_fp32_product_once():
    q = np.array([[127, -1, 3]], dtype=np.int8)
    s = np.array([np.float32(0.1)], dtype=np.float32)
    x = kv.dequantize_kv_int8(q, s)
    want = (q.astype(np.float32) * s[:, None]).astype(np.float16)
    assert x.dtype == np.float16 and np.array_equal(x.view(np.uint16), want.view(np.uint16))


def test_roundtrip_error_bound_of_the_reference_test():
    # src/blackwell_ops/tests/test_kv_quant.py: C, N = 32, 4096, randn fp16, max error < 0.1
    rng = np.random.Generator(np.random.PCG64(3))
    x = rng.standard_normal((32, 4096), dtype=np.float32).astype(np.float16)
    q, s = kv.quantize_kv_int8(x)
    err = np.abs(x.astype(np.float32) - kv.dequantize_kv_int8(q, s).astype(np.float32)).max()
    assert err < 0.1
