"""GPU parity: tcgen05 LoRA delta / merge / fused requantisation vs the oracle.

The oracle reproduces the reference kernels' fp32 accumulator exactly (j-ordered
sums; see oracle/lora.py).  The tensor core sums the same exact products in a
different order, so a delta may differ from the reference by one fp16 ulp when
the fp32 sum lands next to a rounding boundary: the tests require every value
within one ulp of the oracle and count the differing fraction.  Requantisation
is checked bit-exactly as ``quantize_weight_int8(merged)`` of the merged weight
that the same kernels produce, and against the oracle's codes with at most a
handful of +-1 code differences traced to those 1-ulp deltas.
"""
import numpy as np
import pytest

from cases import LORA_CASES
from oracle import inputs, lora, quant
from oracle.numerics import F16

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

QWEN = inputs.QWEN3_06B_PROJ


def dev16(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float16)).to(dev)


def within_ulp(got, want, delta=None):
    """|got - want| <= one fp16 ulp of want.  For merged weights add one ulp of
    the delta: a delta that differs by one ulp changes the exact sum W + delta by
    that much before the sum is rounded (at most one more ulp of the result)."""
    got = np.asarray(got, np.float16).astype(np.float64)
    w16 = np.asarray(want, np.float16)
    ulp = np.spacing(np.abs(w16)).astype(np.float64)
    if delta is not None:
        ulp = ulp + np.spacing(np.abs(np.asarray(delta, np.float16))).astype(np.float64)
    diff = np.abs(got - w16.astype(np.float64))
    assert (diff <= ulp).all(), diff.max()
    return float((diff > 0).mean())


@pytest.fixture(scope="module")
def ops():
    from blackwell_ops import _lib, cuda
    from blackwell_ops.kernels import quantize_weight_int8

    yield cuda, quantize_weight_int8
    assert _lib.device_status() == 0


def make(seed, r, n, k):
    return inputs.lora_a(seed, r, k), inputs.lora_b(seed + 1, n, r), inputs.weight(seed + 2, n, k, F16)


CASES = [(c[1], c[2], c[3], c[4], c[5]) for c in LORA_CASES] + [
    (400 + i, r, n, k, 2.0) for i, (r, (_, k, n)) in enumerate((r, p) for r in (16, 128) for p in QWEN)
] + [(450, 8, 128, 64, 2.0), (451, 64, 130, 136, 1.0), (452, 32, 1, 128, 2.0), (453, 16, 257, 1000, 2.0),
      (454, 12, 50, 100, 2.0), (455, 16, 33, 100, 0.75),  # these two: CUDA-core fallback layouts
      # several tiles per CTA of the persistent kernel, crossing row blocks; a ragged last column tile
      (460, 128, 1024, 8192, 2.0), (461, 16, 2000, 4112, 2.0), (462, 64, 640, 3008, 2.0)]


@pytest.mark.parametrize("seed,r,n,k,s", CASES)
def test_lora_delta(seed, r, n, k, s, cuda_dev, ops):
    cuda, _ = ops
    A, B, _ = make(seed, r, n, k)
    want = lora.lora_delta(A, B, s)
    for fn in (cuda.lora_delta, cuda.lora_delta_tiled):
        got = fn(dev16(A, cuda_dev), dev16(B, cuda_dev), s).cpu().numpy()
        assert within_ulp(got, want) < 0.01
    # the reference test's tolerance (test_lora_ops.py:15)
    ref32 = (B.astype(np.float32) @ A.astype(np.float32)) * s
    assert np.abs(got.astype(np.float32) - ref32).max() < 0.02


@pytest.mark.parametrize("seed,r,n,k,s", CASES)
def test_lora_merge_and_requant(seed, r, n, k, s, cuda_dev, ops):
    cuda, qz = ops
    A, B, W = make(seed, r, n, k)
    Ad, Bd, Wd = dev16(A, cuda_dev), dev16(B, cuda_dev), dev16(W, cuda_dev)
    want = lora.merge(W, A, B, s)
    merged = cuda.lora_merge(Wd, Ad, Bd, s)
    assert within_ulp(merged.cpu().numpy(), want, lora.lora_delta(A, B, s)) < 0.01
    # composition of the two reference ops gives the same bits as the fused merge
    w2 = Wd.clone()
    cuda.add_delta_(w2, cuda.lora_delta(Ad, Bd, s))
    assert torch.equal(w2, merged)
    # in-place merge
    w3 = Wd.clone()
    cuda.lora_merge(w3, Ad, Bd, s, out=w3)
    assert torch.equal(w3, merged)
    # fused requant == quantize(merged) exactly, and == the oracle's quantiser on that merged weight
    q, sc = cuda.lora_merge_requant(Wd, Ad, Bd, s)
    q2, sc2 = qz(merged)
    assert torch.equal(q, q2) and torch.equal(sc, sc2)
    qo, so = quant.quantize_weight_int8(merged.cpu().numpy(), F16)
    assert np.array_equal(q.cpu().numpy(), qo) and np.array_equal(sc.cpu().numpy(), so)
    # against the oracle's own pipeline: codes differ only where a merged value differs by one ulp
    qo2, _, _ = lora.merge_requant(W, A, B, s)
    d = np.abs(q.cpu().numpy().astype(np.int32) - qo2.astype(np.int32))
    assert d.max() <= 1
    assert (d > 0).mean() < 1e-3


def test_add_delta_bit_exact(cuda_dev, ops):
    cuda, _ = ops
    for n, k in ((64, 128), (3, 5), (1024, 1001)):
        W = inputs.weight(11 + n, n, k, F16, std=1.0)
        D = inputs.weight(12 + n, n, k, F16, std=1.0)
        Wd = dev16(W, cuda_dev)
        cuda.add_delta_(Wd, dev16(D, cuda_dev))
        assert np.array_equal(Wd.cpu().numpy(), lora.add_delta(W, D))
    # unaligned views take the scalar path
    Wd = dev16(inputs.weight(1, 1, 1001, F16), cuda_dev)
    Dd = dev16(inputs.weight(2, 1, 1001, F16), cuda_dev)
    a, b = Wd[0, 1:], Dd[0, :1000]
    want = lora.add_delta(a.cpu().numpy(), b.cpu().numpy())
    cuda.add_delta_(a, b)
    assert np.array_equal(a.cpu().numpy(), want)
    # a strided W (a column slice and a transposed view) is updated element for element in
    # logical order, and nothing outside the view changes
    base = dev16(inputs.weight(3, 96, 130, F16), cuda_dev)
    keep = base.clone()
    view = base[:, 2:66]
    D = dev16(inputs.weight(4, 96, 64, F16), cuda_dev)
    want = lora.add_delta(view.cpu().numpy(), D.cpu().numpy())
    cuda.add_delta_(view, D)
    assert np.array_equal(view.cpu().numpy(), want)
    assert torch.equal(base[:, :2], keep[:, :2]) and torch.equal(base[:, 66:], keep[:, 66:])
    wt = dev16(inputs.weight(5, 80, 48, F16), cuda_dev).t()
    D = dev16(inputs.weight(6, 48, 80, F16), cuda_dev)
    want = lora.add_delta(wt.cpu().numpy(), D.cpu().numpy())
    cuda.add_delta_(wt, D)
    assert np.array_equal(wt.cpu().numpy(), want)


def test_lora_errors_match_reference_messages(cuda_dev, ops):
    cuda, _ = ops
    A = torch.randn(16, 128, device=cuda_dev, dtype=torch.float16)
    B = torch.randn(96, 16, device=cuda_dev, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="A and B must be CUDA"):
        cuda.lora_delta(A.cpu(), B)
    with pytest.raises(RuntimeError, match="A and B must be fp16"):
        cuda.lora_delta(A.float(), B)
    with pytest.raises(RuntimeError, match="B must be"):
        cuda.lora_delta(A, B[:, :8])
    with pytest.raises(RuntimeError, match="shape mismatch"):
        cuda.add_delta_(B.clone(), A)
    with pytest.raises(RuntimeError, match="must be fp16"):
        cuda.add_delta_(B.float(), B)


def test_lora_full_size_70b_requant_properties(cuda_dev, ops):
    """Llama-3-70B down-projection shard: K = 28672 (3584 panels over the resident CTAs, two passes)."""
    cuda, qz = ops
    n, k, r = 1024, 28672, 64
    g = torch.Generator(device=cuda_dev).manual_seed(9)
    W = (torch.randn(n, k, generator=g, device=cuda_dev) * 0.02).half()
    A = (torch.randn(r, k, generator=g, device=cuda_dev) / k ** 0.5).half()
    B = (torch.randn(n, r, generator=g, device=cuda_dev) * 0.01).half()
    merged = cuda.lora_merge(W, A, B, 2.0)
    q, sc = cuda.lora_merge_requant(W, A, B, 2.0)
    q2, sc2 = qz(merged)
    assert torch.equal(q, q2) and torch.equal(sc, sc2)
    d = 2.0 * (B.double() @ A.double())
    ref = W.double() + d
    err = (merged.double() - ref).abs()
    # one fp16 rounding of the delta and one of the sum
    assert bool((err <= (ref.abs() + d.abs()) * 2.0 ** -10 + 2.0 ** -24).all())


def test_lora_merge_requant_batched_equals_single(cuda_dev, ops):
    """One batched launch over mixed shapes/ranks gives the single-problem results bit for bit."""
    cuda, _ = ops
    specs = [(16, 2048, 1024), (16, 1024, 1024), (128, 1024, 2048), (64, 3072, 1024), (16, 1024, 3072),
             (128, 130, 1000), (8, 1, 64), (32, 257, 4096), (16, 96, 5000), (12, 40, 72)]
    items = []
    for i, (r, n, k) in enumerate(specs):
        A, B, W = make(600 + i, r, n, k)
        items.append((dev16(W, cuda_dev), dev16(A, cuda_dev), dev16(B, cuda_dev), 2.0 if i % 3 else 0.75))
    outs = cuda.lora_merge_requant_batched(items)
    for (W, A, B, s), (q, sc) in zip(items, outs):
        q1, s1 = cuda.lora_merge_requant(W, A, B, s)
        assert torch.equal(q, q1) and torch.equal(sc, s1)
        qm, sm = quant.quantize_weight_int8(cuda.lora_merge(W, A, B, s).cpu().numpy(), F16)
        assert np.array_equal(q.cpu().numpy(), qm) and np.array_equal(sc.cpu().numpy(), sm)


def test_lora_merge_requant_special_rows(cuda_dev, ops):
    """Rows holding inf, NaN, only zeros or only tiny values take the exact path and match the quantiser."""
    cuda, qz = ops
    r, n, k = 16, 256, 512
    A, B, W = make(700, r, n, k)
    W = W.copy()
    W[3, 17] = np.inf
    W[5, 400] = -np.inf
    W[7, 1] = np.nan
    W[9, :] = 0
    W[11, :] = np.float16(6e-8)   # subnormal row: zero scale after rounding
    W[130, 300] = np.float16(60000.0)  # near the fp16 maximum: the merge may overflow to inf
    W[13, :] = (np.linspace(-1, 1, k) * 3e-4).astype(np.float16)  # subnormal scale: the clamped packed path
    B[9, :] = 0                   # rows 9, 11 and 13 keep their values through the merge
    B[11, :] = 0
    B[13, :] = 0
    Wd, Ad, Bd = dev16(W, cuda_dev), dev16(A, cuda_dev), dev16(B, cuda_dev)
    merged = cuda.lora_merge(Wd, Ad, Bd, 2.0)
    q, sc = cuda.lora_merge_requant(Wd, Ad, Bd, 2.0)
    q2, sc2 = qz(merged)
    assert torch.equal(q, q2)
    assert torch.equal(sc.view(torch.int16), sc2.view(torch.int16))  # NaN scales compare by bits
    qo, so = quant.quantize_weight_int8(merged.cpu().numpy(), F16)
    assert np.array_equal(q.cpu().numpy(), qo)
    assert np.array_equal(sc.cpu().numpy().view(np.uint16), so.view(np.uint16))


def test_lora_merge_requant_many_problems_reuse_workspace(cuda_dev, ops):
    """More than 16 problems: several launches in a row share one workspace.

    Each launch uses the row-maxima set of its barrier generation's parity and
    clears the other; three rounds of two launches reuse each set several times.
    """
    cuda, _ = ops
    specs = [(16 if i % 2 else 64, 128 * (1 + i % 3), 64 * (2 + i % 5)) for i in range(21)]
    items = []
    for i, (r, n, k) in enumerate(specs):
        A, B, W = make(800 + i, r, n, k)
        items.append((dev16(W, cuda_dev), dev16(A, cuda_dev), dev16(B, cuda_dev), 1.5))
    for _ in range(3):
        outs = cuda.lora_merge_requant_batched(items)
        for (W, A, B, s), (q, sc) in zip(items, outs):
            qm, sm = quant.quantize_weight_int8(cuda.lora_merge(W, A, B, s).cpu().numpy(), F16)
            assert np.array_equal(q.cpu().numpy(), qm) and np.array_equal(sc.cpu().numpy(), sm)


# exact=True: the reference's own j-ordered accumulation on the CUDA cores.  Every cfg2 projection
# (Qwen3-0.6B, r in {16, 128}), odd shapes, strided/odd r, and a cfg5 shard (1/8 of the Llama-3-70B
# up projection's rows): delta, merge and requantisation equal the reference pipeline bit for bit.
EXACT_CASES = [(500 + i, r, n, k, 2.0) for i, (r, (_, k, n)) in enumerate((r, p) for r in (16, 128) for p in QWEN)] + [
    (530, 7, 130, 200, 1.5), (531, 12, 50, 101, 2.0), (532, 128, 33, 1000, 0.75), (533, 16, 3584, 8192, 2.0)]


@pytest.mark.parametrize("seed,r,n,k,s", EXACT_CASES)
def test_lora_exact_mode_bit_exact(seed, r, n, k, s, cuda_dev, ops):
    cuda, _ = ops
    A, B, W = make(seed, r, n, k)
    Ad, Bd, Wd = dev16(A, cuda_dev), dev16(B, cuda_dev), dev16(W, cuda_dev)
    want_d = lora.lora_delta(A, B, s)
    got_d = cuda.lora_delta(Ad, Bd, s, exact=True).cpu().numpy()
    assert np.array_equal(got_d.view(np.uint16), want_d.view(np.uint16))
    want_w = lora.add_delta(W, want_d)
    got_w = cuda.lora_merge(Wd, Ad, Bd, s, exact=True).cpu().numpy()
    assert np.array_equal(got_w.view(np.uint16), want_w.view(np.uint16))
    q_want, s_want = quant.quantize_weight_int8(want_w, F16)
    for q, sc in (cuda.lora_merge_requant(Wd, Ad, Bd, s, exact=True),
                  cuda.lora_merge_requant_batched([(Wd, Ad, Bd, s)], exact=True)[0]):
        assert np.array_equal(q.cpu().numpy(), q_want)
        assert np.array_equal(sc.cpu().numpy().view(np.uint16), np.asarray(s_want).view(np.uint16))
    # in place, strided rows of W
    Wbig = dev16(np.concatenate([W, W[:, :8]], axis=1), cuda_dev)
    view = Wbig[:, :k]
    cuda.lora_merge(view, Ad, Bd, s, out=view, exact=True)
    assert np.array_equal(view.cpu().numpy().view(np.uint16), want_w.view(np.uint16))
