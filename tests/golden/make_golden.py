"""Generate golden vectors from the REAL reference implementation.

Run where the reference source tree is importable (it is not on the GPU box):

    REF_SRC=<reference checkout>/src python tests/golden/make_golden.py

It imports the reference's ``blackwell_ops.kernels.quantize_weight_int8``
(``src/blackwell_ops/kernels/int8_gemm.py:63-68``) and evaluates the
reference tests' own CPU expressions for the GEMM
(``src/blackwell_ops/tests/test_int8_gemm.py:17-18``), the LoRA delta
(``src/blackwell_ops/tests/test_lora_ops.py:14``), ``add_delta_``
(``test_lora_ops.py:26``) and the registry's delta
(``src/blackwell_inference/lora/delta_multi.py:59``) on seeded inputs drawn by
``oracle.inputs``.  Outputs go to ``tests/golden/*.npz`` plus a JSON index of
SHA-256 digests for the large cases.  The reference's CUDA / Triton kernels do
not run on CPU, so those are pinned through the reference tests' expressions.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

ref_src = os.environ.get("REF_SRC")
if not ref_src:
    sys.exit("set REF_SRC to the reference's src/ directory")
sys.path.insert(0, ref_src)
sys.dont_write_bytecode = True

import torch  # noqa: E402
from blackwell_ops.kernels import quantize_weight_int8 as ref_quantize  # noqa: E402

from oracle import inputs  # noqa: E402
from oracle.numerics import BF16, F16, F32  # noqa: E402

from cases import EDGE_CASES, GEMM_CASES, LORA_CASES, QUANT_CASES, edge_weight  # noqa: E402


def to_torch(a: np.ndarray, dtype: str) -> torch.Tensor:
    if dtype == BF16:
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)
    return torch.from_numpy(np.ascontiguousarray(a))


def to_numpy(t: torch.Tensor, dtype: str) -> np.ndarray:
    if dtype == BF16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.contiguous().numpy()


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main() -> None:
    index = {"quant": {}, "edge": {}, "gemm": {}, "lora": {}}
    small = {}

    for name, seed, n, k, dt in QUANT_CASES:
        w = inputs.weight(seed, n, k, dt)
        q, s = ref_quantize(to_torch(w, dt))
        qn, sn = q.numpy(), to_numpy(s, dt)
        index["quant"][name] = {"seed": seed, "n": n, "k": k, "dtype": dt,
                                "q_sha256": digest(qn), "scale_sha256": digest(sn)}
        if n * k <= 64 * 1024:
            small[f"quant/{name}/q"] = qn
            small[f"quant/{name}/scale"] = sn
        else:
            small[f"quant/{name}/q_rows"] = qn[:4].copy()
            small[f"quant/{name}/scale_head"] = sn[:64].copy()

    for name, dt in EDGE_CASES:
        w = edge_weight(name, dt)
        q, s = ref_quantize(to_torch(w, dt))
        small[f"edge/{name}/w"] = w
        small[f"edge/{name}/q"] = q.numpy()
        small[f"edge/{name}/scale"] = to_numpy(s, dt)
        index["edge"][name] = {"dtype": dt, "shape": list(w.shape)}

    for name, seed, m, n, k, xdt, wdt in GEMM_CASES:
        x = inputs.activations(seed + 1, m, k, xdt)
        w = inputs.weight(seed, n, k, wdt)
        q, s = ref_quantize(to_torch(w, wdt))
        xt = to_torch(x, xdt)
        # reference test's oracle, test_int8_gemm.py:17-18
        w_deq = q.float() * s.unsqueeze(-1)
        ref = xt.float() @ w_deq.t()
        small[f"gemm/{name}/ref_fp32"] = ref.numpy()
        index["gemm"][name] = {"seed": seed, "m": m, "n": n, "k": k, "x_dtype": xdt, "w_dtype": wdt,
                               "q_sha256": digest(q.numpy())}

    for name, seed, r, n, k, scaling in LORA_CASES:
        A = inputs.lora_a(seed, r, k)
        B = inputs.lora_b(seed + 1, n, r)
        W = inputs.weight(seed + 2, n, k, F16)
        At, Bt, Wt = to_torch(A, F16), to_torch(B, F16), to_torch(W, F16)
        # test_lora_ops.py:14 — fp32 reference of lora_delta, and the fp16 value lora_ops.cu:26 stores
        ref32 = (Bt.float() @ At.float()) * scaling
        delta = ref32.to(torch.float16)
        # test_lora_ops.py:26 — add_delta_ reference
        Wp = (Wt.float() + delta.float()).to(torch.float16)
        q, s = ref_quantize(Wp)
        # delta_multi.py:59 — registry delta, fp16 matmul then * scaling
        reg = (Bt @ At) * scaling
        arrays = {"delta_fp32": ref32.numpy(), "merged": Wp.numpy(), "registry_delta": reg.numpy(),
                  "q": q.numpy(), "scale": s.numpy()}
        entry = {"seed": seed, "r": r, "n": n, "k": k, "scaling": scaling}
        for key, arr in arrays.items():
            entry[f"{key}_sha256"] = digest(arr)
            small[f"lora/{name}/{key}"] = arr if n * k <= 128 * 1024 else arr[:2].copy()
        index["lora"][name] = entry

    np.savez_compressed(HERE / "golden.npz", **small)
    index["generator"] = {"torch": torch.__version__, "numpy": np.__version__,
                          "reference": "blackwell_ops.kernels.quantize_weight_int8 (src/blackwell_ops/kernels/int8_gemm.py:63-68)"}
    (HERE / "golden_index.json").write_text(json.dumps(index, indent=1, sort_keys=True))
    print("wrote", HERE / "golden.npz", (HERE / "golden.npz").stat().st_size, "bytes")


if __name__ == "__main__":
    main()
