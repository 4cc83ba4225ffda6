"""The kernels' fast quantiser path equals the exact (IEEE-division) path.

Compiles tests/quant_fast_check.cpp (a C++ restatement of quant_fast /
quant_one from csrc/quant_math.cuh) and sweeps every finite fp16 / bf16
weight against every 16th positive scale of the dtype, plus a sampled fp32
sweep, and the packed fp16 path (quant4_f16: fp16 clamp and +1536
round-to-integer) the same way.  The clamp-free packed path is swept over every
(w, s) a row can hold when its scale is a normal fp16 number (|w| <= the row
maximum that gives s; 9.3e8 pairs at stride 1).  The full sweep (every scale: 2.0e9 fp16 and 2.1e9 bf16
pairs, the clamp-free sweep and the packed bf16 sweep over 1.9e9 pairs) was run once with stride 1 and also
found no mismatch.
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
                                          ("f16packed_noclamp", 4), ("bf16packed", 16)])
def test_fast_quantiser_matches_exact_division(checker, dtype, stride):
    out = subprocess.run([str(checker), dtype, str(stride)], capture_output=True, text=True, check=True).stdout
    fields = dict(kv.split("=") for kv in out.split())
    assert int(fields["total"]) > 1e8
    assert int(fields["mismatches"]) == 0, out
