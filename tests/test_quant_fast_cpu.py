"""The kernels' fast quantiser paths equal the exact (IEEE-division) path.

Compiles tests/quant_fast_check.cpp (a C++ restatement of quant_fast /
quant_one and of the packed quantisers quant4_f16 / quant4_bf16 from
csrc/quant_math.cuh) and sweeps every finite fp16 / bf16 weight against every
16th positive scale of the dtype, plus a sampled fp32 sweep.  The packed paths
(fp16 clamp and +1536 round-to-integer; bf16 clamp and +1.5 * 2^23) have no
midpoint check or exact-division fix-up at all, so for them these sweeps are the
proof that none is needed: the clamp-free fp16 path is swept here over all 9.3e8
(w, s) pairs a row with a normal fp16 scale can hold (|w| <= the row maximum that
gives s, stride 1), and the full sweeps of the clamped fp16 path (every finite w
and every positive finite s: 2.0e9 pairs) and of the bf16 path (1.9e9 pairs)
were run once at stride 1 and found no mismatch, as did the full scalar sweeps
(2.0e9 fp16 and 2.1e9 bf16 pairs).
"""
import shutil
import subprocess
from pathlib import Path

import pytest

HERE = Path(__file__).resolve().parent


@pytest.fixture(scope="module")
def checker(tmp_path_factory):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    exe = tmp_path_factory.mktemp("qfc") / "quant_fast_check"
    subprocess.run([gxx, "-O2", "-std=c++17", "-ffp-contract=off", "-fno-fast-math", "-pthread",
                    str(HERE / "quant_fast_check.cpp"), "-o", str(exe)], check=True)
    return exe


@pytest.mark.parametrize("dtype,stride", [("f16", 16), ("bf16", 16), ("f32", 1), ("f16packed", 16),
                                          ("f16packed_noclamp", 1), ("bf16packed", 16)])
def test_fast_quantiser_matches_exact_division(checker, dtype, stride):
    out = subprocess.run([str(checker), dtype, str(stride)], capture_output=True, text=True, check=True).stdout
    fields = dict(kv.split("=") for kv in out.split())
    assert int(fields["total"]) > 1e8
    assert int(fields["mismatches"]) == 0, out
