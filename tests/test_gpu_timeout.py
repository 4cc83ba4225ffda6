"""Bounded device waits run out into an error, not a hang (one GPU, no fault).

The fused all-gather GEMM waits for its peers' output words in its own
signal-pad mailbox.  Here rank 0 of a "world" of two is launched alone: no
rank 1 ever sends, so rank 0's wait must run out.  With the wait
limit set to 20 ms the kernel returns, the device status records the wait
site, ``blackwell_ops.device.check`` raises ``DeviceTimeoutError`` (a
``RuntimeError``), and the device stays usable: a plain GEMM afterwards still
matches the fp32 reference.  Nothing here traps, faults or hangs the GPU.
"""
import ctypes

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

SITE_RECEIVE = 131  # the wait for a peer's mailbox words


def test_wait_limit_roundtrip(cuda_dev):
    from blackwell_ops import device

    old = device.wait_limit(cuda_dev)
    try:
        device.set_wait_limit(0.05, cuda_dev)
        assert abs(device.wait_limit(cuda_dev) - 0.05) < 1e-6
    finally:
        device.set_wait_limit(old, cuda_dev)
    assert abs(device.wait_limit(cuda_dev) - old) < 1e-6


def test_gather_peer_that_never_arrives_raises(cuda_dev):
    from blackwell_ops import _lib, device
    from blackwell_ops.kernels import int8_gemm

    lib = _lib.lib
    torch.cuda.set_device(cuda_dev)
    g = torch.Generator(device=cuda_dev).manual_seed(7)
    m, n, k = 16, 256, 2048
    x = torch.randn(m, k, generator=g, device=cuda_dev).half()
    q = torch.randint(-127, 128, (n, k), generator=g, device=cuda_dev, dtype=torch.int8)
    s = (torch.rand(n, generator=g, device=cuda_dev) * 1e-3 + 1e-4).half()
    y = torch.zeros(m, 2 * n, dtype=torch.float16, device=cuda_dev)
    nbytes = lib.bw_w8a16_gemm_allgather_signal_bytes(m, n, 2)
    sigs = [torch.zeros(nbytes // 4, dtype=torch.int32, device=cuda_dev) for _ in range(2)]
    need = lib.bw_w8a16_gemm_allgather_workspace_size(m, n, k)
    ws = torch.zeros(max(need, 16), dtype=torch.uint8, device=cuda_dev)
    sp = (ctypes.c_void_p * 2)(*[t.data_ptr() for t in sigs])
    assert device.status(cuda_dev, clear=True) == 0
    old = device.wait_limit(cuda_dev)
    device.set_wait_limit(0.02, cuda_dev)
    try:
        rc = lib.bw_w8a16_gemm_allgather(x.data_ptr(), 0, k, q.data_ptr(), k, s.data_ptr(), 0, y.data_ptr(), 2 * n,
                                         0, m, n, k, sp, nbytes, 2, 0, ws.data_ptr(), ws.numel(),
                                         _lib.stream_ptr(cuda_dev))
        assert rc == 0, lib.bw_last_error()
        with pytest.raises(device.DeviceTimeoutError) as err:
            device.check(cuda_dev, "int8_gemm (all-gather)")
        assert isinstance(err.value, RuntimeError)
        assert err.value.site == SITE_RECEIVE
        assert "timed out" in str(err.value)
        assert device.status(cuda_dev) == 0  # check() cleared it
    finally:
        device.set_wait_limit(old, cuda_dev)
    # the context is intact: a plain GEMM on the same stream is still right
    y = int8_gemm(x, q, s)
    ref = x.float() @ (q.float() * s.float()[:, None]).t()
    assert float((y.float() - ref).abs().max()) <= 1e-2
    assert device.status(cuda_dev) == 0
