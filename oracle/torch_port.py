"""The reference's CPU PyTorch path for this hot path (test/benchmark infrastructure only).

These are the reference's own torch expressions, run on CPU tensors.  They are
what ``bench.py`` times as the CPU baseline (``cpu_baseline``, kind "port")
and as ``--impl reference``; they are never the product path.

* ``quantize_weight_int8`` - ``src/blackwell_ops/kernels/int8_gemm.py:63-68``.
* ``int8_gemm``            - the reference test's dequantise-then-matmul,
  ``src/blackwell_ops/tests/test_int8_gemm.py:17-18``, cast to x.dtype the way
  ``int8_gemm`` returns it (``int8_gemm.py:82``).
* ``lora_delta``           - ``(B.float() @ A.float()) * scaling`` rounded to
  fp16 (``src/blackwell_ops/tests/test_lora_ops.py:14``, the value
  ``lora_ops.cu:26`` stores).
* ``add_delta_``           - ``W.float() + delta.float()`` rounded to fp16
  (``test_lora_ops.py:26``; ``lora_ops.cu:36``).
* ``merge_requant``        - ``lora_delta`` -> ``add_delta_`` ->
  ``quantize_weight_int8``.
"""
from __future__ import annotations

import torch


def quantize_weight_int8(w: torch.Tensor):
    w_abs_max = w.abs().amax(dim=-1, keepdim=True).clamp(min=1e-8)
    scale = w_abs_max / 127.0
    w_int8 = (w / scale).round().clamp(-127, 127).to(torch.int8)
    return w_int8, scale.squeeze(-1)


def int8_gemm(x: torch.Tensor, w_int8: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    w_deq = w_int8.float() * scale.float().unsqueeze(-1)
    return (x.float() @ w_deq.t()).to(x.dtype)


def lora_delta(A: torch.Tensor, B: torch.Tensor, scaling: float = 1.0) -> torch.Tensor:
    return ((B.float() @ A.float()) * scaling).to(torch.float16)


def add_delta_(W: torch.Tensor, delta: torch.Tensor) -> None:
    W.copy_((W.float() + delta.float()).to(W.dtype))


def merge_requant(W: torch.Tensor, A: torch.Tensor, B: torch.Tensor, scaling: float):
    Wp = W.clone()
    add_delta_(Wp, lora_delta(A, B, scaling))
    return quantize_weight_int8(Wp)
