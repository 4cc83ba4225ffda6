"""LoRA delta operators for B200 (drop-in for ``src/blackwell_ops/cuda/__init__.py``).

Same names, arguments and error behaviour as the reference's CUDA extension
for this path:

* ``lora_delta(A, B, scaling)``        reference ``cuda/__init__.py:89`` -> ``lora_ops.cu:43-60``
* ``lora_delta_tiled(A, B, scaling)``  reference ``cuda/__init__.py:99`` -> ``lora_tiled.cu:88-103``
* ``add_delta_(W, delta)``             reference ``cuda/__init__.py:94`` -> ``lora_ops.cu:62-71``

Both delta variants run the same tcgen05 kernel here (the reference's two
kernels compute the same value).  Fused additions:

* ``lora_merge(W, A, B, scaling, out=None)`` = ``add_delta_(W.clone(), lora_delta(A, B, scaling))``
  without materialising the delta (``out=W`` merges in place).
* ``lora_merge_requant(W, A, B, scaling)`` = ``quantize_weight_int8`` of that
  merged weight, which is never written to memory.

Errors are ``RuntimeError`` with the reference's TORCH_CHECK messages.
Kernels run on torch's current stream (the reference used the legacy default
stream).
"""
from __future__ import annotations

import torch

from .._lib import RequantProblem, check, lib, stream_ptr

_ws: dict[tuple[int, int], torch.Tensor] = {}


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor | None:
    """Requantisation scratch (grid barrier + two sets of row maxima) per (device, stream).

    Zeroed once at allocation and always passed with its full size: each call
    clears the set of row maxima the next call uses.  A larger need replaces it
    with a new zeroed buffer.
    """
    if nbytes == 0:
        return None
    key = (device.index if device.index is not None else torch.cuda.current_device(), stream_ptr(device))
    ws = _ws.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _ws[key] = ws
    return ws


def reset_workspaces() -> None:
    """Zero every cached requantisation workspace (needed only after a device-side timeout, which
    can leave a grid barrier or a set of row maxima mid-way)."""
    for ws in _ws.values():
        ws.zero_()


def _check_ab(A: torch.Tensor, B: torch.Tensor) -> tuple[int, int, int]:
    if not (A.is_cuda and B.is_cuda):
        raise RuntimeError("A and B must be CUDA")
    if A.dtype != torch.float16 or B.dtype != torch.float16:
        raise RuntimeError("A and B must be fp16")
    if A.dim() != 2 or B.dim() != 2:
        raise RuntimeError("A and B must be 2D")
    r, K = A.shape
    N = B.shape[0]
    if B.shape[1] != r:
        raise RuntimeError("B must be [N, r]")
    if A.device != B.device:
        raise RuntimeError("A and B must be on the same device")
    return r, K, N


def lora_delta(A: torch.Tensor, B: torch.Tensor, scaling: float = 1.0, exact: bool = False) -> torch.Tensor:
    """A: [r, K], B: [N, r] -> delta: [N, K] = B @ A * scaling (fp16, fp32 accumulation).

    ``exact=True`` sums on the CUDA cores in the reference kernels' j order, so the result equals
    the reference bit for bit (the tensor-core default is within one fp16 ulp, < 1 % of values
    differing)."""
    r, K, N = _check_ab(A, B)
    A = A.contiguous()
    B = B.contiguous()
    delta = torch.empty((N, K), dtype=torch.float16, device=A.device)
    if N and K:
        if r == 0:
            return delta.zero_()
        with torch.cuda.device(A.device):
            fn = lib.bw_lora_delta_exact if exact else lib.bw_lora_delta
            check(fn(A.data_ptr(), B.data_ptr(), delta.data_ptr(), N, K, r, float(scaling), stream_ptr(A.device)),
                  "lora_delta")
    return delta


def lora_delta_tiled(A: torch.Tensor, B: torch.Tensor, scaling: float = 1.0, exact: bool = False) -> torch.Tensor:
    """A: [r, K], B: [N, r] -> delta: [N, K] = B @ A * scaling (same kernel as lora_delta)"""
    return lora_delta(A, B, scaling, exact=exact)


def add_delta_(W: torch.Tensor, delta: torch.Tensor) -> None:
    """W += delta, in-place (fp16(fp32 W + fp32 delta)), element i of W with element i of delta
    in logical (row-major) order.

    The reference's checks (lora_ops.cu:62-66: CUDA, fp16, equal numel) are the only ones.  A
    non-contiguous W is updated through a contiguous copy written back into the view (the
    reference kernel walks W's storage from its first element instead, which for a strided view
    pairs the wrong elements and writes outside the view).
    """
    if not (W.is_cuda and delta.is_cuda):
        raise RuntimeError("W and delta must be CUDA")
    if W.dtype != torch.float16 or delta.dtype != torch.float16:
        raise RuntimeError("must be fp16")
    if W.numel() != delta.numel():
        raise RuntimeError("shape mismatch")
    if not W.numel():
        return
    delta = delta.contiguous()
    target = W if W.is_contiguous() else W.contiguous()
    with torch.cuda.device(W.device):
        check(lib.bw_add_delta(target.data_ptr(), delta.data_ptr(), W.numel(), stream_ptr(W.device)), "add_delta_")
    if target is not W:
        W.copy_(target)


def _check_w(W: torch.Tensor, N: int, K: int) -> torch.Tensor:
    if not W.is_cuda:
        raise RuntimeError("W must be CUDA")
    if W.dtype != torch.float16:
        raise RuntimeError("W must be fp16")
    if W.dim() != 2 or tuple(W.shape) != (N, K):
        raise RuntimeError(f"W must be [N, K] = [{N}, {K}]")
    return W if W.stride(1) == 1 else W.contiguous()


def lora_merge(W: torch.Tensor, A: torch.Tensor, B: torch.Tensor, scaling: float = 1.0,
               out: torch.Tensor | None = None, exact: bool = False) -> torch.Tensor:
    """W' = fp16(W + fp16(B @ A * scaling)); ``out=W`` merges in place.  ``exact=True``: the
    reference's j-ordered accumulation on the CUDA cores (bit-exact with add_delta_(W, lora_delta))."""
    r, K, N = _check_ab(A, B)
    W = _check_w(W, N, K)
    A = A.contiguous()
    B = B.contiguous()
    if out is None:
        out = torch.empty((N, K), dtype=torch.float16, device=W.device)
    elif out.shape != W.shape or out.dtype != torch.float16 or out.stride(1) != 1:
        raise RuntimeError("out must be an fp16 [N, K] tensor with unit column stride")
    if N and K:
        if r == 0:
            if out.data_ptr() != W.data_ptr():
                out.copy_(W)
            return out
        with torch.cuda.device(W.device):
            fn = lib.bw_lora_merge_exact if exact else lib.bw_lora_merge
            check(fn(W.data_ptr(), W.stride(0), A.data_ptr(), B.data_ptr(), float(scaling), out.data_ptr(),
                     out.stride(0), N, K, r, stream_ptr(W.device)), "lora_merge")
    return out


def lora_merge_requant(W: torch.Tensor, A: torch.Tensor, B: torch.Tensor, scaling: float = 1.0,
                       exact: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
    """(w_int8, scale) = quantize_weight_int8(lora_merge(W, A, B, scaling)), fused.

    ``exact=True`` merges with the reference's j-ordered accumulation on the CUDA cores into a
    temporary fp16 weight and quantises that, so codes and scales equal the reference pipeline
    (``quantize_weight_int8(add_delta_(W, lora_delta(A, B, s)))``) bit for bit."""
    r, K, N = _check_ab(A, B)
    W = _check_w(W, N, K)
    if K == 0:
        raise RuntimeError("lora_merge_requant: Expected reduction dim -1 to have non-zero size")
    if exact:
        from ..kernels import quantize_weight_int8

        return quantize_weight_int8(lora_merge(W, A, B, scaling, exact=True))
    A = A.contiguous()
    B = B.contiguous()
    q = torch.empty((N, K), dtype=torch.int8, device=W.device)
    scale = torch.empty((N,), dtype=torch.float16, device=W.device)
    if N == 0:
        return q, scale
    if r == 0:
        from ..kernels import quantize_weight_int8

        return quantize_weight_int8(W)
    nbytes = lib.bw_lora_merge_requant_workspace_size(N, K, r)
    ws = _workspace(W.device, nbytes)
    with torch.cuda.device(W.device):
        check(lib.bw_lora_merge_requant(W.data_ptr(), W.stride(0), A.data_ptr(), B.data_ptr(), float(scaling),
                                        q.data_ptr(), K, scale.data_ptr(), N, K, r,
                                        ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
                                        stream_ptr(W.device)),
              "lora_merge_requant")
    return q, scale


def lora_merge_requant_batched(items, exact: bool = False):
    """Fused merge + requantisation of several projections in as few launches as possible.

    ``items``: iterable of ``(W, A, B, scaling)`` on one device.  Returns a list
    of ``(w_int8, scale)``, each equal to ``lora_merge_requant(W, A, B, scaling, exact)``.
    """
    items = list(items)
    if not items:
        return []
    if exact:
        return [lora_merge_requant(W, A, B, s, exact=True) for W, A, B, s in items]
    keep, outs, probs = [], [], []
    dev = None
    for W, A, B, scaling in items:
        r, K, N = _check_ab(A, B)
        W = _check_w(W, N, K)
        if K == 0:
            raise RuntimeError("lora_merge_requant: Expected reduction dim -1 to have non-zero size")
        if dev is None:
            dev = W.device
        elif W.device != dev:
            raise RuntimeError("lora_merge_requant_batched: all problems must be on one device")
        A = A.contiguous()
        B = B.contiguous()
        q = torch.empty((N, K), dtype=torch.int8, device=dev)
        sc = torch.empty((N,), dtype=torch.float16, device=dev)
        outs.append((q, sc))
        if N == 0:
            continue
        if r == 0:
            from ..kernels import quantize_weight_int8

            q2, s2 = quantize_weight_int8(W)
            q.copy_(q2)
            sc.copy_(s2)
            continue
        keep.append((W, A, B))
        probs.append(RequantProblem(W.data_ptr(), W.stride(0), A.data_ptr(), B.data_ptr(), float(scaling),
                                    q.data_ptr(), K, sc.data_ptr(), N, K, r))
    if probs:
        arr = (RequantProblem * len(probs))(*probs)
        nbytes = lib.bw_lora_merge_requant_batched_workspace_size(arr, len(probs))
        ws = _workspace(dev, nbytes)
        with torch.cuda.device(dev):
            check(lib.bw_lora_merge_requant_batched(arr, len(probs), ws.data_ptr() if ws is not None else None,
                                                    ws.numel() if ws is not None else 0, stream_ptr(dev)),
                  "lora_merge_requant_batched")
    return outs


def _norm_check(x: torch.Tensor, weight: torch.Tensor, residual: torch.Tensor | None) -> None:
    tensors = (x, weight) if residual is None else (x, residual, weight)
    if not all(t.is_cuda for t in tensors):
        raise RuntimeError("inputs must be CUDA" if residual is not None else "x and w must be CUDA")
    if x.dim() != 2:
        raise RuntimeError("x must be [M, N]")
    if x.dtype not in (torch.float16, torch.bfloat16) or any(t.dtype != x.dtype for t in tensors):
        raise RuntimeError("x, residual and weight must share one dtype, fp16 or bf16")
    if weight.numel() != x.shape[1] or (residual is not None and residual.shape != x.shape):
        raise RuntimeError("shape mismatch")


def fused_residual_rmsnorm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                           eps: float = 1e-6) -> torch.Tensor:
    """rmsnorm(x + residual) * weight, x and residual [M, N] (reference ``cuda/__init__.py:64-67``,
    kernel ``basic_ops.cu:49-78``): fp32 sum, the reference's summation order, IEEE fp32."""
    _norm_check(x, weight, residual)
    return _norm(x, residual, weight, eps)


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """rmsnorm(x) * weight, x [M, N] (reference ``cuda/__init__.py:60-61``, ``basic_ops.cu:16-46``)."""
    _norm_check(x, weight, None)
    return _norm(x, None, weight, eps)


def _norm(x, residual, weight, eps):
    from .._lib import DTYPE_CODE

    x = x.contiguous()
    residual = residual.contiguous() if residual is not None else None
    weight = weight.contiguous()
    M, N = x.shape
    out = torch.empty_like(x)
    if M and N:
        with torch.cuda.device(x.device):
            check(lib.bw_residual_rmsnorm(x.data_ptr(), residual.data_ptr() if residual is not None else None,
                                          DTYPE_CODE[x.dtype], N, weight.data_ptr(), float(eps), out.data_ptr(), N,
                                          M, N, stream_ptr(x.device)), "fused_residual_rmsnorm")
    return out


def quantize_kv_int8(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """x: [C, N] fp16 -> (q [C, N] int8, scale [C] fp32), per-channel symmetric.

    scale = max|x_row| / 127 in fp32 (NaN elements ignored); q = clamp(lrint(x / scale), -127, 127).
    Reference: quantize_kv_int8, src/blackwell_ops/cuda/kv_quant.cu:17-42, 62-76.
    """
    if not (x.is_cuda and x.dtype == torch.float16):
        raise RuntimeError("x must be CUDA fp16")
    if x.dim() != 2:
        raise RuntimeError("x must be [C, N]")
    if x.stride(1) != 1:
        x = x.contiguous()
    C, N = x.shape
    q = torch.empty((C, N), dtype=torch.int8, device=x.device)
    scale = torch.empty((C,), dtype=torch.float32, device=x.device)
    if C:
        with torch.cuda.device(x.device):
            check(lib.bw_quantize_kv_int8(x.data_ptr(), C, N, x.stride(0), q.data_ptr(), N, scale.data_ptr(),
                                          stream_ptr(x.device)), "quantize_kv_int8")
    return q, scale


def dequantize_kv_int8(q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """q: [C, N] int8, scale: [C] fp32 -> x [C, N] fp16 = fp16(q * scale[:, None]).

    Reference: dequantize_kv_int8, src/blackwell_ops/cuda/kv_quant.cu:47-58, 78-90.
    """
    if not (q.is_cuda and q.dtype == torch.int8):
        raise RuntimeError("q must be CUDA int8")
    if not (scale.is_cuda and scale.dtype == torch.float32):
        raise RuntimeError("scale must be CUDA fp32")
    if q.dim() != 2:
        raise RuntimeError("q must be [C, N]")
    if q.stride(1) != 1:
        q = q.contiguous()
    C, N = q.shape
    if scale.numel() < C:
        raise RuntimeError("scale must hold one value per channel")
    scale = scale.contiguous()
    x = torch.empty((C, N), dtype=torch.float16, device=q.device)
    if C and N:
        with torch.cuda.device(q.device):
            check(lib.bw_dequantize_kv_int8(q.data_ptr(), q.stride(0), scale.data_ptr(), C, N, x.data_ptr(), N,
                                            stream_ptr(q.device)), "dequantize_kv_int8")
    return x


__all__ = ["lora_delta", "lora_delta_tiled", "add_delta_", "lora_merge", "lora_merge_requant",
           "lora_merge_requant_batched", "quantize_kv_int8", "dequantize_kv_int8", "fused_residual_rmsnorm", "rmsnorm"]
