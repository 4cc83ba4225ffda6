"""GPU: the grouped W8A16 GEMM (one launch over up to four GEMMs that share x).

Each output must meet the GEMM bar against the dequantise-matmul in fp64 (fp16: max |err| <= 1e-2
and relative <= 1e-3; bf16: |err| <= 1e-2 + 2^-8 |ref|) and stay within one output ulp (plus the
fp32 accumulation bound) of the separate ``int8_gemm`` call, whose split-K pieces may be summed in
another grouping.  Shapes: a Qwen3-0.6B layer's q/k/v (2048, 1024, 1024) and gate/up (3072, 3072)
at M = 1, 16, 64; ragged N (1000, 3, 129, 4096); a Llama-3-70B up projection split in four.
"""
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

CASES = [(1, 1024, (2048, 1024, 1024), torch.float16), (16, 1024, (2048, 1024, 1024), torch.float16),
         (64, 1024, (3072, 3072), torch.bfloat16), (16, 1024, (3072, 3072), torch.bfloat16),
         (5, 520, (1000, 3, 129, 4096), torch.float16), (16, 8192, (7168, 7168, 7168, 7168), torch.bfloat16)]


def _problem(g, dev, n, k, dt):
    from blackwell_ops.kernels import quantize_weight_int8

    w = (torch.randn(n, k, generator=g, device=dev) * 0.02).to(dt)
    return quantize_weight_int8(w)


@pytest.mark.parametrize("m,k,ns,dt", CASES)
def test_grouped_matches_separate_and_reference(cuda_dev, m, k, ns, dt):
    from blackwell_ops import _lib
    from blackwell_ops.kernels import int8_gemm, int8_gemm_grouped

    g = torch.Generator(device=cuda_dev).manual_seed(m + k + sum(ns))
    x = torch.randn(m, k, generator=g, device=cuda_dev).to(dt)
    probs = [_problem(g, cuda_dev, n, k, dt) for n in ns]
    ys = int8_gemm_grouped(x, probs)
    ys2 = int8_gemm_grouped(x, probs)
    for (q, s), y, y2 in zip(probs, ys, ys2):
        assert y.shape == (m, q.shape[0]) and torch.equal(y, y2)  # deterministic
        ref = x.double() @ (q.double() * s.double()[:, None]).t()
        err = (y.double() - ref).abs()
        if dt == torch.float16:
            assert float(err.max()) <= 1e-2 and float(err.norm() / ref.norm()) <= 1e-3
        else:
            assert bool((err <= 1e-2 + 2.0 ** -8 * ref.abs()).all())
        sep = int8_gemm(x, q, s)
        ulp = 2.0 ** (-10 if dt == torch.float16 else -7)
        acc = 2.0 ** -20 * (x.double().abs() @ (q.double().abs() * s.double()[:, None]).t())
        assert bool(((y.double() - sep.double()).abs() <= ulp * ref.abs() + acc + 1e-6).all())
    assert _lib.device_status() == 0


def test_grouped_rejects_bad_groups(cuda_dev):
    from blackwell_ops.kernels import int8_gemm_grouped

    x = torch.randn(4, 64, device=cuda_dev, dtype=torch.float16)
    q = torch.zeros(8, 64, device=cuda_dev, dtype=torch.int8)
    s = torch.ones(8, device=cuda_dev, dtype=torch.float16)
    with pytest.raises(RuntimeError):
        int8_gemm_grouped(x, [])
    with pytest.raises(RuntimeError):
        int8_gemm_grouped(x, [(q, s)] * 5)
    with pytest.raises(RuntimeError):
        int8_gemm_grouped(x, [(q[:, :32], s)])
    y, = int8_gemm_grouped(x, [(q, s)])  # one problem: the plain GEMM
    assert y.shape == (4, 8) and float(y.abs().max()) == 0.0
