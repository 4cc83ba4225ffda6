"""The W8A16 GEMM entry point that allocates nothing (bw_w8a16_gemm_noalloc).

Some callers cannot give the library device memory (a serving runtime whose
memory manager owns the whole GPU, a foreign-language binding with no CUDA
allocator), so this entry point keeps its split-K scratch in a fixed array
inside libbw_ops.so.  This test calls it through the C ABI, on two calls in a
row, for shapes whose plan does use that scratch, and checks that

* it returns exactly the bits of the workspace-taking bw_w8a16_gemm (the
  kernel, its plan and its k-ordered reduction are the same, so the result is
  deterministic), and
* it meets the GEMM tolerance against the fp32 oracle (max |err| <= 1e-2,
  relative <= 1e-3 against the float64-accumulated dequantise-then-matmul),

and that shapes needing more scratch than the array are refused.  It lives in
its own file, collected last, and needs nothing from other tests.
"""
import numpy as np
import pytest

from oracle import gemm, inputs, quant
from oracle.numerics import F16

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

# every shape here plans split-K or stream-K pieces, i.e. needs scratch
SHAPES = [(16, 1024, 4096), (1, 1024, 4096), (16, 2048, 1024), (48, 2048, 2048), (64, 3584, 8192), (16, 151936, 1024)]


def _gemm_with_workspace(lib, st, x, q, s, m, n, k):
    need = lib.bw_w8a16_gemm_workspace_size(m, n, k)
    ws = torch.zeros(max(need, 16), dtype=torch.uint8, device=x.device)
    y = torch.empty(m, n, dtype=x.dtype, device=x.device)
    rc = lib.bw_w8a16_gemm(x.data_ptr(), 0, k, q.data_ptr(), k, s.data_ptr(), 0, y.data_ptr(), n, m, n, k,
                           ws.data_ptr(), ws.numel(), st)
    assert rc == 0, lib.bw_last_error()
    return y, need


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_noalloc_matches_workspace_entry_point_and_oracle(m, n, k):
    from blackwell_ops import _lib

    lib = _lib.lib
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    st = _lib.stream_ptr(dev)
    w = inputs.weight(m * 7 + n + k, n, k, F16)
    qn, sn = quant.quantize_weight_int8(w, F16)
    xn = inputs.activations(m + k, m, k, F16)
    x = torch.from_numpy(xn).to(dev)
    q = torch.from_numpy(qn).to(dev)
    s = torch.from_numpy(sn).to(dev)
    ref, need = _gemm_with_workspace(lib, st, x, q, s, m, n, k)
    assert 0 < need <= lib.bw_w8a16_gemm_static_scratch_bytes(), need
    want = gemm.exact(xn, F16, qn, sn, F16)
    for _ in range(2):
        y = torch.full((m, n), float("nan"), dtype=torch.float16, device=dev)
        rc = lib.bw_w8a16_gemm_noalloc(x.data_ptr(), 0, k, q.data_ptr(), k, s.data_ptr(), 0, y.data_ptr(), n, m, n,
                                       k, st)
        assert rc == 0, lib.bw_last_error()
        torch.cuda.synchronize()
        assert torch.equal(y.view(torch.int16), ref.view(torch.int16)), "differs from bw_w8a16_gemm"
        got = y.float().cpu().numpy().astype(np.float64)
        err = np.abs(got - want)
        assert err.max() <= 1e-2, err.max()
        assert np.linalg.norm(got - want) / np.linalg.norm(want) <= 1e-3
    assert _lib.device_status() == 0


def test_noalloc_rejects_shapes_beyond_its_scratch():
    from blackwell_ops import _lib

    lib = _lib.lib
    dev = torch.device("cuda:0")
    limit = lib.bw_w8a16_gemm_static_scratch_bytes()
    candidates = [(m, n, k) for m in (128, 96, 64) for n in (8192, 4096, 2048) for k in (65536, 131072, 262144)]
    over = [c for c in candidates if lib.bw_w8a16_gemm_workspace_size(*c) > limit]
    assert over, "no candidate shape needs more split-K scratch than the static array"
    m, n, k = min(over, key=lambda c: c[0] * c[2] + c[1] * c[2])
    x = torch.zeros(m, k, dtype=torch.float16, device=dev)
    q = torch.zeros(n, k, dtype=torch.int8, device=dev)
    s = torch.ones(n, dtype=torch.float16, device=dev)
    y = torch.empty(m, n, dtype=torch.float16, device=dev)
    rc = lib.bw_w8a16_gemm_noalloc(x.data_ptr(), 0, k, q.data_ptr(), k, s.data_ptr(), 0, y.data_ptr(), n, m, n, k,
                                   _lib.stream_ptr(dev))
    assert rc == _lib.BW_ERR_WORKSPACE
    assert b"static array" in lib.bw_last_error()
