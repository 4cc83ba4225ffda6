"""CPU checks of the C-ABI library: it loads without a GPU and exports every
symbol ``include/bw_ops.h`` declares (no compute calls)."""
import ctypes
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    text = (ROOT / "include" / "bw_ops.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(bw_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_api():
    syms = declared_symbols()
    for name in ("bw_quantize_rowwise_int8", "bw_w8a16_gemm", "bw_lora_delta", "bw_add_delta", "bw_lora_merge",
                 "bw_lora_merge_requant", "bw_status_string", "bw_device_status"):
        assert name in syms


def test_library_exports_every_declared_symbol():
    from blackwell_ops import _lib

    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing
    assert set(declared_symbols()) == set(_lib.SIGNATURES)


def test_host_only_entry_points():
    from blackwell_ops import _lib

    lib = _lib.lib
    assert lib.bw_version() >= 10000
    assert lib.bw_status_string(0) == b"ok"
    assert lib.bw_status_string(4) == b"device wait timed out"
    # argument validation happens before any device call
    assert lib.bw_quantize_rowwise_int8(None, 0, 4, 0, 0, None, 0, None, None) == _lib.BW_ERR_INVALID_ARGUMENT
    assert b"k >= 1" in lib.bw_last_error()
    assert lib.bw_w8a16_gemm(None, 2, 8, None, 8, None, 0, None, 8, 1, 1, 8, None, 0, None) == _lib.BW_ERR_INVALID_ARGUMENT
    assert lib.bw_lora_delta(None, None, None, 4, 4, 0, 1.0, None) == _lib.BW_ERR_INVALID_ARGUMENT
    assert lib.bw_add_delta(None, None, -1, None) == _lib.BW_ERR_INVALID_ARGUMENT
    # empty problems are no-ops that never touch the device
    assert lib.bw_w8a16_gemm(None, 0, 8, None, 8, None, 0, None, 8, 0, 0, 8, None, 0, None) == 0


def test_gemm_workspace_contract_host_only():
    """Workspace planning is host-only: the zeroed counter prefix has one size (4 KB) for every
    split shape, plans without split tiles need no workspace, stream-K plans of decode tiles keep
    two fp32 pieces per CTA, and the fused SwiGLU op plans 64-column tiles."""
    from blackwell_ops import _lib

    lib = _lib.lib
    shapes = [(16, 1024, 4096), (16, 1024, 3072), (16, 151936, 1024), (16, 28672, 8192), (64, 3072, 8192)]
    for m, n, k in shapes:
        need = lib.bw_w8a16_gemm_workspace_size(m, n, k)
        zeroed = lib.bw_w8a16_gemm_workspace_zeroed_bytes(m, n, k)
        assert need > 0 and zeroed == 4096 and need % 16 == 0, (m, n, k, need, zeroed)
    # one CTA per tile with the whole K: no pieces, no counters (prefill; and a small decode GEMM,
    # which runs on at most 32 CTAs)
    assert lib.bw_w8a16_gemm_workspace_size(16, 3072, 1024) == 0
    assert lib.bw_w8a16_gemm_workspace_size(2048, 14336, 4096) == 0
    assert lib.bw_w8a16_gemm_workspace_zeroed_bytes(2048, 14336, 4096) == 0
    # LM head at M=16: stream-K over 148 CTAs, two 128 x 16 fp32 pieces per CTA after the counters
    sms = lib.bw_w8a16_gemm_workspace_size(16, 151936, 1024) - 4096
    assert sms % (2 * 128 * 16 * 4) == 0 and sms // (2 * 128 * 16 * 4) >= 100
    assert lib.bw_w8a16_gemm_swiglu_workspace_size(16, 3072, 1024) > 0
    assert lib.bw_w8a16_gemm_swiglu_workspace_size(0, 3072, 1024) == 0
    # argument checks of the fused op happen before any device call
    assert lib.bw_w8a16_gemm_swiglu(None, 2, 8, None, None, 8, None, None, 0, None, 8, 1, 1, 8, None, 0,
                                    None) == _lib.BW_ERR_INVALID_ARGUMENT
