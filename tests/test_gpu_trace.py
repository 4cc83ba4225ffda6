"""GPU: the device-side phase trace (``blackwell_ops.device.Trace``).

One traced call each of the W8A16 GEMM and of the fused merge + requantisation: every CTA
claims a record, the phases a launch passes through are stamped in order, and tracing leaves
the results unchanged (the same outputs as an untraced call) and the device status clear.
"""
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _one(tr, kernel):
    ls = [l for l in tr.launches() if l.kernel == kernel]
    assert len(ls) == 1, [l.kernel for l in tr.launches()]
    return ls[0]


def test_trace_gemm_phases(cuda_dev):
    from blackwell_ops import _lib
    from blackwell_ops.device import PHASES, Trace
    from blackwell_ops.kernels import int8_gemm, quantize_weight_int8

    g = torch.Generator(device=cuda_dev).manual_seed(5)
    x = torch.randn(16, 4096, generator=g, device=cuda_dev).half()
    q, s = quantize_weight_int8((torch.randn(2048, 4096, generator=g, device=cuda_dev) * 0.02).half())
    y0 = int8_gemm(x, q, s)
    with Trace(records=1024, device=cuda_dev) as tr:
        y1 = int8_gemm(x, q, s)
    assert torch.equal(y0, y1)
    l = _one(tr, "w8a16_persistent")
    assert l.phases == PHASES and l.stamps.shape == (l.ctas, len(PHASES))
    assert bool((l.stamps[:, 0] > 0).all())  # every CTA started
    ph = l.phases_us()
    assert 0.0 <= ph["first_tile"] <= ph["epilogue_done"]
    assert _lib.device_status() == 0


def test_trace_requant_phases(cuda_dev):
    from blackwell_ops import _lib
    from blackwell_ops.cuda import lora_merge_requant
    from blackwell_ops.device import REQUANT_PHASES, Trace

    g = torch.Generator(device=cuda_dev).manual_seed(6)
    n, k, r = 1024, 2048, 16
    W = (torch.randn(n, k, generator=g, device=cuda_dev) * 0.02).half()
    A = (torch.randn(r, k, generator=g, device=cuda_dev) / k ** 0.5).half()
    B = (torch.randn(n, r, generator=g, device=cuda_dev) * 0.01).half()
    q0, s0 = lora_merge_requant(W, A, B, 2.0)
    with Trace(records=1024, device=cuda_dev) as tr:
        q1, s1 = lora_merge_requant(W, A, B, 2.0)
    assert torch.equal(q0, q1) and torch.equal(s0, s1)
    l = _one(tr, "lora_requant_coop")
    assert l.phases == REQUANT_PHASES
    st = l.stamps
    assert bool((st > 0).all())  # every CTA passed every phase
    # per CTA, each pair stamped in this order (by one thread, or across a barrier)
    for a, b in ((0, 1), (1, 2), (2, 3), (2, 4), (3, 5), (4, 5), (0, 6), (6, 7), (8, 9)):
        assert bool((st[:, b] >= st[:, a]).all()), (REQUANT_PHASES[a], REQUANT_PHASES[b])
    # the barrier opens only after the last CTA arrived
    assert int(st[:, 3].min()) >= int(st[:, 2].max())
    ph = l.phases_us()
    assert ph["pass2_done"] >= ph["barrier_passed"] >= ph["pass1_done"]
    assert _lib.device_status() == 0
