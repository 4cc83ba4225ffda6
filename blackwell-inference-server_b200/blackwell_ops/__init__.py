"""blackwell_ops (B200 edition): the W8A16 GEMM and LoRA-delta operators of
blackwell-ops, re-implemented as hand-written sm_100a CUDA kernels behind a
C ABI (``include/bw_ops.h``).

Drop-in names, as in the reference package:

* ``blackwell_ops.kernels.quantize_weight_int8``, ``blackwell_ops.kernels.int8_gemm``
  (reference ``src/blackwell_ops/kernels/int8_gemm.py``)
* ``blackwell_ops.cuda.lora_delta``, ``lora_delta_tiled``, ``add_delta_``
  (reference ``src/blackwell_ops/cuda/__init__.py:89-101``)

plus the fused ``blackwell_ops.cuda.lora_merge`` / ``lora_merge_requant`` and
the column-parallel ``blackwell_ops.nsplit`` wrapper.
"""

__version__ = "0.1.0+b200"
