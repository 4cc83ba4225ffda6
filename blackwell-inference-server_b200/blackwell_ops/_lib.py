"""ctypes binding of libbw_ops.so, the sm_100a C-ABI library (``include/bw_ops.h``).

There is no fallback: if the shared library is missing or fails to load, the
import raises, and every operator raises if a call returns a non-OK status.
Build the library with ``python blackwell-inference-server_b200/csrc/build.py``
(``__graft_entry__.build()`` does it too).
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

LIB_PATH = Path(os.environ.get("BW_OPS_LIB", Path(__file__).resolve().parent / "_lib" / "libbw_ops.so"))

BW_OK = 0
BW_ERR_INVALID_ARGUMENT = 1
BW_ERR_WORKSPACE = 2
BW_ERR_CUDA = 3
BW_ERR_DEVICE_TIMEOUT = 4
BW_ERR_UNSUPPORTED = 5

GATHER_MAX_M = 256  # largest m of the fused all-gather GEMM (include/bw_ops.h)

DTYPE_CODE = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}

# Every symbol declared in include/bw_ops.h, with its ctypes signature.
_c = ctypes
_P = _c.c_void_p
_I64 = _c.c_int64


class RequantProblem(ctypes.Structure):
    """Mirror of bw_lora_requant_problem (include/bw_ops.h)."""

    _fields_ = [("w", _P), ("ldw", _I64), ("a", _P), ("b", _P), ("scaling", _c.c_float), ("q", _P),
                ("ldq", _I64), ("scale", _P), ("n", _I64), ("k", _I64), ("r", _I64)]


SIGNATURES = {
    "bw_status_string": (_c.c_char_p, [_c.c_int]),
    "bw_last_error": (_c.c_char_p, []),
    "bw_version": (_c.c_int, []),
    "bw_quantize_rowwise_int8": (_c.c_int, [_P, _c.c_int, _I64, _I64, _I64, _P, _I64, _P, _P]),
    "bw_w8a16_gemm_workspace_size": (_c.c_size_t, [_I64, _I64, _I64]),
    "bw_w8a16_gemm_workspace_zeroed_bytes": (_c.c_size_t, [_I64, _I64, _I64]),
    "bw_w8a16_gemm": (_c.c_int, [_P, _c.c_int, _I64, _P, _I64, _P, _c.c_int, _P, _I64, _I64, _I64, _I64, _P,
                                 _c.c_size_t, _P]),
    "bw_w8a16_gemm_swiglu_workspace_size": (_c.c_size_t, [_I64, _I64, _I64]),
    "bw_w8a16_gemm_swiglu": (_c.c_int, [_P, _c.c_int, _I64, _P, _P, _I64, _P, _P, _c.c_int, _P, _I64, _I64, _I64,
                                        _I64, _P, _c.c_size_t, _P]),
    "bw_w8a16_gemm_static_scratch_bytes": (_c.c_size_t, []),
    "bw_w8a16_gemm_noalloc": (_c.c_int, [_P, _c.c_int, _I64, _P, _I64, _P, _c.c_int, _P, _I64, _I64, _I64, _I64,
                                         _P]),
    "bw_w8a16_gemm_grouped_workspace_size": (_c.c_size_t, [_I64, _P, _c.c_int, _I64]),
    "bw_w8a16_gemm_grouped": (_c.c_int, [_P, _c.c_int, _I64, _c.c_int, _P, _P, _P, _c.c_int, _P, _P, _P, _I64, _I64,
                                         _P, _c.c_size_t, _P]),
    "bw_w8a16_gemm_allgather_workspace_size": (_c.c_size_t, [_I64, _I64, _I64]),
    "bw_w8a16_gemm_allgather_signal_bytes": (_c.c_size_t, [_I64, _I64, _c.c_int]),
    "bw_w8a16_gemm_allgather": (_c.c_int, [_P, _c.c_int, _I64, _P, _I64, _P, _c.c_int, _P, _I64, _I64, _I64, _I64,
                                           _I64, _c.POINTER(_c.c_void_p), _c.c_size_t, _c.c_int, _c.c_int, _P,
                                           _c.c_size_t, _P]),
    "bw_debug_streamk_walk": (_c.c_int, [_I64, _I64, _c.c_int, _c.c_int, _P, _c.c_int]),
    "bw_debug_streamk_start": (_I64, [_I64, _I64, _c.c_int, _c.c_int]),
    "bw_debug_streamk_owner": (_c.c_int, [_I64, _I64, _c.c_int, _I64]),
    "bw_debug_streamk_pieces": (_c.c_int, [_I64, _I64, _c.c_int, _c.c_int, _P]),
    "bw_lora_delta": (_c.c_int, [_P, _P, _P, _I64, _I64, _I64, _c.c_float, _P]),
    "bw_add_delta": (_c.c_int, [_P, _P, _I64, _P]),
    "bw_lora_delta_exact": (_c.c_int, [_P, _P, _P, _I64, _I64, _I64, _c.c_float, _P]),
    "bw_lora_merge_exact": (_c.c_int, [_P, _I64, _P, _P, _c.c_float, _P, _I64, _I64, _I64, _I64, _P]),
    "bw_lora_merge": (_c.c_int, [_P, _I64, _P, _P, _c.c_float, _P, _I64, _I64, _I64, _I64, _P]),
    "bw_lora_merge_requant_workspace_size": (_c.c_size_t, [_I64, _I64, _I64]),
    "bw_lora_merge_requant": (_c.c_int, [_P, _I64, _P, _P, _c.c_float, _P, _I64, _P, _I64, _I64, _I64, _P,
                                         _c.c_size_t, _P]),
    "bw_lora_merge_requant_batched_workspace_size": (_c.c_size_t, [_c.POINTER(RequantProblem), _c.c_int]),
    "bw_lora_merge_requant_batched": (_c.c_int, [_c.POINTER(RequantProblem), _c.c_int, _P, _c.c_size_t, _P]),
    "bw_device_status": (_c.c_int, [_c.c_int, _c.POINTER(_c.c_int), _P]),
    "bw_residual_rmsnorm": (_c.c_int, [_P, _P, _c.c_int, _I64, _P, _c.c_float, _P, _I64, _I64, _I64, _P]),
    "bw_w8a16_gemm_rmsnorm_workspace_size": (_c.c_size_t, [_I64, _I64, _I64]),
    "bw_w8a16_gemm_rmsnorm": (_c.c_int, [_P, _P, _c.c_int, _I64, _P, _c.c_float, _P, _I64, _P, _c.c_int, _P, _I64,
                                         _I64, _I64, _I64, _P, _c.c_size_t, _P]),
    "bw_quantize_kv_int8": (_c.c_int, [_P, _I64, _I64, _I64, _P, _I64, _P, _P]),
    "bw_dequantize_kv_int8": (_c.c_int, [_P, _I64, _P, _I64, _I64, _P, _I64, _P]),
    "bw_set_wait_limit_ns": (_c.c_int, [_c.c_uint64]),
    "bw_get_wait_limit_ns": (_c.c_int, [_c.POINTER(_c.c_uint64)]),
    "bw_trace_enable": (_c.c_int, [_P, _c.c_size_t]),
    "bw_trace_records": (_c.c_int, [_c.POINTER(_c.c_uint)]),
}


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"libbw_ops.so not found at {LIB_PATH}; build it with "
            "`python blackwell-inference-server_b200/csrc/build.py` (no CPU fallback exists)"
        )
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


class BwError(RuntimeError):
    """A libbw_ops call returned a non-OK status (a RuntimeError, like TORCH_CHECK)."""

    def __init__(self, status: int, op: str):
        self.status = status
        detail = lib.bw_last_error().decode(errors="replace")
        super().__init__(f"{op}: {lib.bw_status_string(status).decode()}: {detail}")


def check(status: int, op: str) -> None:
    if status != BW_OK:
        raise BwError(status, op)


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def device_status(clear: bool = True, device: torch.device | None = None) -> int:
    """Synchronise and return the device-side status (0 = no bounded wait expired)."""
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    detail = ctypes.c_int(0)
    with torch.cuda.device(dev):
        st = lib.bw_device_status(1 if clear else 0, ctypes.byref(detail), stream_ptr(dev))
    if st not in (BW_OK, BW_ERR_DEVICE_TIMEOUT):
        check(st, "device_status")
    return detail.value


def require_cuda(*tensors: torch.Tensor, msg: str) -> None:
    for t in tensors:
        if not t.is_cuda:
            raise RuntimeError(msg)
