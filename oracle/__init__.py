"""CPU oracle for the W8A16 GEMM / LoRA delta / merge / requantisation path.

TEST INFRASTRUCTURE ONLY.  Nothing in the shipped package imports this
directory; only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
legs of ``bench.py`` use it, and there only as the checker (or, in
``bench.py --impl reference`` and ``cpu_baseline``, as the timed stand-in for
the reference's own CPU PyTorch path).

Modules
-------
``numerics``   fp16 / bf16 round-to-nearest-even helpers on numpy arrays.
``quant``      restatement of ``quantize_weight_int8``
               (reference ``src/blackwell_ops/kernels/int8_gemm.py:63-68``).
``gemm``       dequantise-then-matmul oracle for ``int8_gemm``
               (reference ``src/blackwell_ops/kernels/int8_gemm.py:15-60`` and
               ``src/blackwell_ops/tests/test_int8_gemm.py:17-18``).
``lora``       ``lora_delta`` / ``lora_delta_tiled`` / ``add_delta_`` and the
               merged pipeline (reference ``src/blackwell_ops/cuda/lora_ops.cu``,
               ``src/blackwell_ops/cuda/lora_tiled.cu``).
``kv``         the KV-cache per-channel quantiser and dequantiser
               (reference ``src/blackwell_ops/cuda/kv_quant.cu:17-58``).
``norm``       residual + RMSNorm in the reference kernel's summation order
               (reference ``src/blackwell_ops/cuda/basic_ops.cu:16-78``).
``inputs``     seeded synthetic inputs shared by the golden-vector script,
               the tests and the benchmarks.
``torch_port`` the reference's CPU PyTorch expressions, verbatim in meaning,
               used for CPU-baseline timing.

Parity pin: ``tests/golden/make_golden.py`` imports the real reference
(``blackwell_ops.kernels.quantize_weight_int8`` and the reference tests'
dequantise-matmul / ΔW expressions) and records its outputs; the CPU test
suite checks this oracle against those fixtures bit for bit.
"""
