"""INT8 weight-only (W8A16) GEMM and per-channel int8 quantiser for B200.

Drop-in for ``src/blackwell_ops/kernels/int8_gemm.py`` of the reference:

* ``quantize_weight_int8(w)`` (reference ``:63-68``) -> ``(w_int8, scale)``,
  bit-exact with the reference, computed by ``bw_quantize_rowwise_int8``.
* ``int8_gemm(x, w_int8, scale)`` (reference ``:71-107``) -> ``y = x @ (w_int8 * scale).T``
  in x.dtype with fp32 accumulation, computed by the tcgen05 kernel behind
  ``bw_w8a16_gemm``.

Both run on torch's current CUDA stream and allocate outputs with the caching
allocator, as the reference does.  Split-K scratch is a per-(device, stream)
workspace kept by this module; make one warm-up call before capturing a CUDA
graph so the workspace exists.
"""
from __future__ import annotations

import threading

import torch

from .._lib import DTYPE_CODE, check, lib, stream_ptr

_ws_lock = threading.Lock()
_workspaces: dict[tuple[int, int], torch.Tensor] = {}


def _workspace(device: torch.device, stream: int, nbytes: int) -> torch.Tensor | None:
    """Per-(device, stream) split-K workspace; counters start (and stay) zero."""
    if nbytes == 0:
        return None
    key = (device.index if device.index is not None else torch.cuda.current_device(), stream)
    with _ws_lock:
        ws = _workspaces.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            _workspaces[key] = ws
        return ws


def reset_workspaces() -> None:
    """Zero every cached workspace (needed only after a device-side timeout)."""
    with _ws_lock:
        for ws in _workspaces.values():
            ws.zero_()


def quantize_weight_int8(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-output-channel symmetric int8 quantization.

    ``w`` [..., K] fp16 / bf16 / fp32 on a CUDA device.  Returns ``w_int8``
    (same shape, int8) and ``scale`` (``w.shape[:-1]``, w.dtype) with
    ``scale = max|w_row| / 127`` (clamped >= 1e-8) and
    ``w_int8 = clamp(round(w / scale), -127, 127)``, rounded exactly as the
    reference rounds them.
    """
    if not w.is_cuda:
        raise RuntimeError("quantize_weight_int8: w must be a CUDA tensor")
    if w.dtype not in DTYPE_CODE:
        raise RuntimeError(f"quantize_weight_int8: unsupported dtype {w.dtype}")
    if w.dim() == 0:
        raise RuntimeError("quantize_weight_int8: w must have at least one dimension")
    k = w.shape[-1]
    if k == 0:
        raise RuntimeError("quantize_weight_int8: Expected reduction dim -1 to have non-zero size")
    lead = tuple(w.shape[:-1])
    w2 = w.reshape(-1, k)
    if w2.stride(-1) != 1:
        w2 = w2.contiguous()
    n = w2.shape[0]
    q = torch.empty((n, k), dtype=torch.int8, device=w.device)
    scale = torch.empty((n,), dtype=w.dtype, device=w.device)
    if n:
        with torch.cuda.device(w.device):
            check(
                lib.bw_quantize_rowwise_int8(w2.data_ptr(), DTYPE_CODE[w.dtype], n, k, w2.stride(0), q.data_ptr(), k,
                                             scale.data_ptr(), stream_ptr(w.device)),
                "quantize_weight_int8",
            )
    return q.reshape(*lead, k), scale.reshape(lead)


def int8_gemm(x: torch.Tensor, w_int8: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """
    x: [M, K] fp16 / bf16
    w_int8: [N, K] int8
    scale: [N] fp16 / bf16 / fp32
    returns: [M, N] in x.dtype
    """
    if not (x.is_cuda and w_int8.is_cuda and scale.is_cuda):
        raise RuntimeError("int8_gemm: x, w_int8 and scale must be CUDA tensors")
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise RuntimeError(f"int8_gemm: x must be fp16 or bf16, got {x.dtype}")
    if w_int8.dtype != torch.int8:
        raise RuntimeError(f"int8_gemm: w_int8 must be int8, got {w_int8.dtype}")
    if scale.dtype not in DTYPE_CODE:
        raise RuntimeError(f"int8_gemm: unsupported scale dtype {scale.dtype}")
    if x.dim() != 2 or w_int8.dim() != 2:
        raise RuntimeError("int8_gemm: x must be [M, K] and w_int8 [N, K]")
    M, K = x.shape
    N = w_int8.shape[0]
    if w_int8.shape[1] != K:
        raise RuntimeError(f"int8_gemm: K mismatch ({K} vs {w_int8.shape[1]})")
    if scale.numel() != N:
        raise RuntimeError(f"int8_gemm: scale must have N={N} elements")
    y = torch.empty(M, N, device=x.device, dtype=x.dtype)
    if M == 0 or N == 0:
        return y
    if K == 0:
        return y.zero_()
    if x.stride(1) != 1 or x.stride(0) < K:
        x = x.contiguous()
    if w_int8.stride(1) != 1 or w_int8.stride(0) < K:
        w_int8 = w_int8.contiguous()
    scale = scale.reshape(N)
    if scale.stride(0) != 1:
        scale = scale.contiguous()
    with torch.cuda.device(x.device):
        st = stream_ptr(x.device)
        nbytes = lib.bw_w8a16_gemm_workspace_size(M, N, K)
        ws = _workspace(x.device, st, nbytes)
        check(
            lib.bw_w8a16_gemm(x.data_ptr(), DTYPE_CODE[x.dtype], x.stride(0), w_int8.data_ptr(), w_int8.stride(0),
                              scale.data_ptr(), DTYPE_CODE[scale.dtype], y.data_ptr(), N, M, N, K,
                              ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0, st),
            "int8_gemm",
        )
    return y


def int8_gemm_swiglu(x: torch.Tensor, w_gate: torch.Tensor, s_gate: torch.Tensor, w_up: torch.Tensor,
                     s_up: torch.Tensor) -> torch.Tensor:
    """Fused ``swiglu(int8_gemm(x, w_gate, s_gate), int8_gemm(x, w_up, s_up))`` in one launch.

    The MLP's gate and up projections share x; one kernel streams both int8 weights, rounds each
    product to x.dtype as int8_gemm would, and writes ``silu(g) * u`` (fp32 silu, as the reference
    swiglu kernel, src/blackwell_ops/cuda/basic_ops.cu:112-122).  Same argument rules as int8_gemm;
    w_gate and w_up are [N, K], s_gate and s_up [N] of one dtype.  Returns [M, N] in x.dtype.
    """
    if not all(t.is_cuda for t in (x, w_gate, s_gate, w_up, s_up)):
        raise RuntimeError("int8_gemm_swiglu: all inputs must be CUDA tensors")
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise RuntimeError(f"int8_gemm_swiglu: x must be fp16 or bf16, got {x.dtype}")
    if w_gate.dtype != torch.int8 or w_up.dtype != torch.int8:
        raise RuntimeError("int8_gemm_swiglu: w_gate and w_up must be int8")
    if s_gate.dtype not in DTYPE_CODE or s_up.dtype != s_gate.dtype:
        raise RuntimeError("int8_gemm_swiglu: s_gate and s_up must share one supported dtype")
    if x.dim() != 2 or w_gate.dim() != 2 or w_up.shape != w_gate.shape:
        raise RuntimeError("int8_gemm_swiglu: x must be [M, K], w_gate and w_up [N, K]")
    M, K = x.shape
    N = w_gate.shape[0]
    if w_gate.shape[1] != K:
        raise RuntimeError(f"int8_gemm_swiglu: K mismatch ({K} vs {w_gate.shape[1]})")
    if s_gate.numel() != N or s_up.numel() != N:
        raise RuntimeError(f"int8_gemm_swiglu: scales must have N={N} elements")
    y = torch.empty(M, N, device=x.device, dtype=x.dtype)
    if M == 0 or N == 0:
        return y
    if K == 0:
        return y.zero_()
    if x.stride(1) != 1 or x.stride(0) < K:
        x = x.contiguous()
    w_gate = w_gate.contiguous()
    w_up = w_up.contiguous()
    s_gate = s_gate.reshape(N).contiguous()
    s_up = s_up.reshape(N).contiguous()
    with torch.cuda.device(x.device):
        st = stream_ptr(x.device)
        nbytes = lib.bw_w8a16_gemm_swiglu_workspace_size(M, N, K)
        ws = _workspace(x.device, st, nbytes)
        check(
            lib.bw_w8a16_gemm_swiglu(x.data_ptr(), DTYPE_CODE[x.dtype], x.stride(0), w_gate.data_ptr(),
                                     w_up.data_ptr(), K, s_gate.data_ptr(), s_up.data_ptr(), DTYPE_CODE[s_gate.dtype],
                                     y.data_ptr(), N, M, N, K, ws.data_ptr() if ws is not None else None,
                                     ws.numel() if ws is not None else 0, st),
            "int8_gemm_swiglu",
        )
    return y


def int8_gemm_grouped(x: torch.Tensor, weights) -> list[torch.Tensor]:
    """``[int8_gemm(x, w_i, s_i) for (w_i, s_i) in weights]`` in one launch (up to 4 GEMMs sharing x,
    e.g. a layer's q/k/v or gate/up projections): the persistent kernel's schedule spans the union of
    their output tiles, so the small projections stream as one weight walk.  Each result meets the
    int8_gemm tolerance; split-K pieces may be summed in another grouping than in separate calls.
    """
    import ctypes

    weights = [(w, s) for w, s in weights]
    if not 1 <= len(weights) <= 4:
        raise RuntimeError("int8_gemm_grouped: 1 to 4 (w_int8, scale) pairs")
    if not x.is_cuda or x.dtype not in (torch.float16, torch.bfloat16) or x.dim() != 2:
        raise RuntimeError("int8_gemm_grouped: x must be a 2-D fp16 / bf16 CUDA tensor")
    M, K = x.shape
    sdt = weights[0][1].dtype
    ws_, ss, ys = [], [], []
    for w, s in weights:
        if not (w.is_cuda and s.is_cuda) or w.dtype != torch.int8 or w.dim() != 2 or w.shape[1] != K:
            raise RuntimeError("int8_gemm_grouped: every w_int8 must be a CUDA int8 [N, K] tensor with x's K")
        if s.dtype != sdt or s.dtype not in DTYPE_CODE or s.numel() != w.shape[0]:
            raise RuntimeError("int8_gemm_grouped: scales must share one dtype and have N elements")
        ws_.append(w if w.stride(1) == 1 and w.stride(0) >= K else w.contiguous())
        ss.append(s.reshape(-1).contiguous())
        ys.append(torch.empty(M, w.shape[0], device=x.device, dtype=x.dtype))
    if M == 0 or K == 0 or any(w.shape[0] == 0 for w in ws_):
        return [int8_gemm(x, w, s) for w, s in weights]
    if x.stride(1) != 1 or x.stride(0) < K:
        x = x.contiguous()
    c = len(ws_)

    def ptrs(ts):
        return (ctypes.c_void_p * c)(*[t.data_ptr() for t in ts])

    def i64(vals):
        return (ctypes.c_int64 * c)(*vals)

    n = i64([w.shape[0] for w in ws_])
    with torch.cuda.device(x.device):
        st = stream_ptr(x.device)
        nbytes = lib.bw_w8a16_gemm_grouped_workspace_size(M, n, c, K)
        wsp = _workspace(x.device, st, nbytes)
        check(lib.bw_w8a16_gemm_grouped(x.data_ptr(), DTYPE_CODE[x.dtype], x.stride(0), c, ptrs(ws_),
                                        i64([w.stride(0) for w in ws_]), ptrs(ss), DTYPE_CODE[sdt], ptrs(ys),
                                        i64([y.shape[1] for y in ys]), n, M, K,
                                        wsp.data_ptr() if wsp is not None else None,
                                        wsp.numel() if wsp is not None else 0, st), "int8_gemm_grouped")
    return ys


def int8_gemm_rmsnorm(x: torch.Tensor, residual: torch.Tensor | None, norm_weight: torch.Tensor,
                      w_int8: torch.Tensor, scale: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """``int8_gemm(fused_residual_rmsnorm(x, residual, norm_weight, eps), w_int8, scale)`` in one call.

    The residual + RMSNorm prologue (reference ``src/blackwell_ops/cuda/basic_ops.cu:49-78``;
    ``residual=None`` is plain RMSNorm, ``:16-46``) normalises the rows into the GEMM's workspace
    and the W8A16 GEMM follows with programmatic dependent launch, so its weight stream overlaps the
    normalisation.  Bit-identical to the two ops called one after the other.  x / residual [M, K]
    and norm_weight [K] share x's dtype (fp16 / bf16); w_int8 [N, K]; scale [N]; returns [M, N].
    """
    tensors = [x, norm_weight, w_int8, scale] + ([residual] if residual is not None else [])
    if not all(t.is_cuda for t in tensors):
        raise RuntimeError("int8_gemm_rmsnorm: all inputs must be CUDA tensors")
    if x.dtype not in (torch.float16, torch.bfloat16) or norm_weight.dtype != x.dtype or (
            residual is not None and residual.dtype != x.dtype):
        raise RuntimeError("int8_gemm_rmsnorm: x, residual and norm_weight must share fp16 or bf16")
    if w_int8.dtype != torch.int8 or scale.dtype not in DTYPE_CODE:
        raise RuntimeError("int8_gemm_rmsnorm: w_int8 must be int8 and scale fp16 / bf16 / fp32")
    if x.dim() != 2 or w_int8.dim() != 2 or w_int8.shape[1] != x.shape[1] or norm_weight.numel() != x.shape[1]:
        raise RuntimeError("int8_gemm_rmsnorm: x must be [M, K], norm_weight [K] and w_int8 [N, K]")
    if residual is not None and residual.shape != x.shape:
        raise RuntimeError("int8_gemm_rmsnorm: residual must match x")
    M, K = x.shape
    N = w_int8.shape[0]
    if scale.numel() != N:
        raise RuntimeError(f"int8_gemm_rmsnorm: scale must have N={N} elements")
    x = x.contiguous()
    residual = residual.contiguous() if residual is not None else None
    w_int8 = w_int8.contiguous()
    scale = scale.reshape(N).contiguous()
    norm_weight = norm_weight.contiguous()
    y = torch.empty(M, N, device=x.device, dtype=x.dtype)
    if M == 0 or N == 0:
        return y
    with torch.cuda.device(x.device):
        st = stream_ptr(x.device)
        nbytes = lib.bw_w8a16_gemm_rmsnorm_workspace_size(M, N, K)
        ws = _workspace(x.device, st, nbytes)
        check(lib.bw_w8a16_gemm_rmsnorm(x.data_ptr(), residual.data_ptr() if residual is not None else None,
                                        DTYPE_CODE[x.dtype], K, norm_weight.data_ptr(), float(eps), w_int8.data_ptr(),
                                        K, scale.data_ptr(), DTYPE_CODE[scale.dtype], y.data_ptr(), N, M, N, K,
                                        ws.data_ptr(), ws.numel(), st), "int8_gemm_rmsnorm")
    return y
