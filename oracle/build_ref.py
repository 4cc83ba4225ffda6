"""Build the reference's own CUDA operators for sm_100a as a GPU-side checker (test infrastructure only).

    python oracle/build_ref.py

Compiles, from where they lie in the reference tree, the four CUDA sources of the
reference extension that this path's operators replace or sit beside
(``src/blackwell_ops/cuda/{basic_ops,kv_quant,lora_ops,lora_tiled}.cu``), with the
reference loader's own flags (``-O3 --use_fast_math``, ``cuda/__init__.py:48-55``)
except the architecture (sm_100a instead of sm_120), plus ``ref_stubs.cpp`` for the
two operators of its pybind table that need CUTLASS or other sources.  The module
``bw_ref_ops`` lands in ``oracle/_ref/`` (git-ignored; it travels with the tree to a
GPU box).  Only GPU tests import it, as the checker.  Without the reference tree
(e.g. on a GPU box) this does nothing.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
REF_CUDA = Path(os.environ.get("BW_REFERENCE_ROOT", "/root/reference")) / "src" / "blackwell_ops" / "cuda"
SOURCES = ("basic_ops.cu", "kv_quant.cu", "lora_ops.cu", "lora_tiled.cu")


def build(verbose: bool = False) -> Path | None:
    if not all((REF_CUDA / s).exists() for s in SOURCES):
        return None
    from torch.utils.cpp_extension import load

    OUT.mkdir(exist_ok=True)
    load(name="bw_ref_ops", sources=[str(REF_CUDA / s) for s in SOURCES] + [str(HERE / "ref_stubs.cpp")],
         extra_cuda_cflags=["-O3", "--use_fast_math", "-gencode=arch=compute_100a,code=sm_100a"],
         build_directory=str(OUT), verbose=verbose)
    so = next(OUT.glob("bw_ref_ops*.so"), None)
    return so


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
