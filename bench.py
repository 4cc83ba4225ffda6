"""Benchmark harness (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload cfg5|cfg1|cfg2|cfg3|cfg3g|cfg4|quant|delta|merge] [--m M]

Workloads (synthetic seeded data, weights random-init):

  cfg5 (default)  Llama-3-70B MLP W8A16 decode (8192->28672, 28672->8192), M=16 tokens,
        bf16, with 32 adapter int8 copies (merged and requantised at set-up, not
        timed); a step serves one adapter (round robin, 470 MB of int8 weights per
        step > L2).  Column-parallel N-split over the N GPUs: each rank streams its
        1/N of the rows and the output slices are all-gathered inside the GEMM
        epilogue over NVLink peer memory (--gather fused, default) or by NCCL
        (--gather nccl).  Strong scaling.  Metric: GB/s of the whole job (the
        metric's lead quantity, W8A16 decode GEMM vs HBM).
  cfg2  LoRA delta -> merge -> per-channel int8 requantisation
        at the Qwen3-0.6B layer shapes: 7 projections x r in {16, 128}, alpha = 2r
        (scaling 2).  One step merges one decoder layer's 7 projections for both
        adapters; successive steps walk 28 distinct layers (412 MB of fp16
        weights), so every step reads weights that are not in L2.  Metric: delta
        TFLOPS (2 r N K per projection); the kernel is HBM-bound, so the roofline
        is reported in GB/s.  N GPUs: each rank merges its own layers (weak scaling,
        no collective on the data path).
  cfg1  W8A16 GEMM X[16,1024] x W[3072,1024]^T (the reference's CPU-runnable case),
        rotating over 64 weight copies (> L2).  Metric GB/s.
  cfg3  decode sweep over the Qwen3-0.6B linear stack: 28 layers x 7 projections
        + LM head 1024->151936, M tokens (default 16).  Metric GB/s.
  cfg3g  the same sweep with each layer's q/k/v and gate/up as grouped launches that
        share their input (bw_w8a16_gemm_grouped): 4 launches per layer.  GB/s.
  cfg4  prefill W8A16 at Llama-3-8B MLP shapes (4096->14336, 14336->4096), bf16,
        M tokens (default 2048).  Metric TFLOPS.
  quant  quantize_weight_int8 of the Llama-3-8B MLP weights (bf16), GB/s.
  delta / merge  lora_delta / lora_merge at the Llama-3-70B MLP shapes, r = --rank
        (default 128), ΔW TFLOPS with the roofline in GB/s.

--trace adds "phases": device-side globaltimer stamps of a few replayed steps
(per GEMM launch: CTA start spread, first weight tile landed, last MMA done,
epilogue done, all-gather handshake done, gap to the next launch), so the JSON
line names the phase that bounds a step.

Timing: W untimed warm-up steps, then exactly K steps between a barrier +
synchronize on both sides, CUDA events on the launching stream, max over ranks.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
SRC = ROOT / "blackwell-inference-server_b200"
for _p in (str(ROOT), str(SRC)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

QWEN = (("q_proj", 1024, 2048), ("k_proj", 1024, 1024), ("v_proj", 1024, 1024), ("o_proj", 2048, 1024),
        ("gate_proj", 1024, 3072), ("up_proj", 1024, 3072), ("down_proj", 3072, 1024))
LLAMA8B_MLP = ((4096, 14336), (14336, 4096))
LLAMA70B_MLP = ((8192, 28672), (28672, 8192))
QWEN_LAYERS = 28
LM_HEAD = (1024, 151936)


# ---------------------------------------------------------------------------
# environment helpers
# ---------------------------------------------------------------------------
def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def upload_graph(g, stream) -> bool:
    """Upload an instantiated CUDA graph to the device ahead of its first launch (cuGraphUpload), so
    the timed launch does not pay for it.  Returns False where the driver call is unavailable."""
    try:
        import ctypes

        cu = ctypes.CDLL("libcuda.so.1")
        rc = cu.cuGraphUpload(ctypes.c_void_p(g.raw_cuda_graph_exec()), ctypes.c_void_p(stream.cuda_stream))
        torch.cuda.synchronize()
        return rc == 0
    except (OSError, AttributeError, RuntimeError):
        return False


def load_traffic(kernel: str, workload: str):
    p = ROOT / "profiles" / "ncu_traffic.json"
    if not p.exists():
        return None
    try:
        d = json.loads(p.read_text())
        return d.get(f"{kernel}@{workload}")
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi sampler running only while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def gpu_index(local_rank: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v for v in vis.split(",") if v.strip()]
        if local_rank < len(ids) and ids[local_rank].strip().isdigit():
            return int(ids[local_rank])
    return local_rank


# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------
def randn(shape, std, dtype, gen, dev):
    return (torch.randn(shape, generator=gen, device=dev, dtype=torch.float32) * std).to(dtype)


class MergeRequantWorkload:
    """cfg2: LoRA delta + merge + requant for one Qwen3-0.6B layer, r in {16, 128}, per step."""

    name = "cfg2"
    kernel = "lora_requant_coop_kernel"
    unit = "TFLOPS"
    metric_kind = "tflops"
    ranks_r = (16, 128)

    def __init__(self, dev, rank, world, layers=QWEN_LAYERS):
        from blackwell_ops import _lib

        self.lib = _lib.lib
        self.dev = dev
        self.rank = rank
        self.layers = layers
        g = torch.Generator(device=dev).manual_seed(1000 + rank)
        self.W, self.A, self.B, self.Q, self.S = [], [], [], [], []
        for _ in range(layers):
            self.W.append([randn((n, k), 0.02, torch.float16, g, dev) for _, k, n in QWEN])
            self.A.append({r: [randn((r, k), 1.0 / math.sqrt(k), torch.float16, g, dev) for _, k, n in QWEN]
                           for r in self.ranks_r})
            self.B.append({r: [randn((n, r), 0.01, torch.float16, g, dev) for _, k, n in QWEN] for r in self.ranks_r})
            self.Q.append({r: [torch.empty((n, k), dtype=torch.int8, device=dev) for _, k, n in QWEN]
                           for r in self.ranks_r})
            self.S.append({r: [torch.empty((n,), dtype=torch.float16, device=dev) for _, k, n in QWEN]
                           for r in self.ranks_r})
        self.flops = sum(2.0 * r * n * k for r in self.ranks_r for _, k, n in QWEN)
        self.bytes = sum(2 * n * k + 2 * r * (n + k) + n * k + 2 * n for r in self.ranks_r for _, k, n in QWEN)
        # one batched call per layer: both adapters' 7 projections (14 problems) in one launch,
        # the two adapters of a projection side by side so the second read of the base weight
        # follows the first (an L2 hit)
        from blackwell_ops._lib import RequantProblem

        self.nprob = len(QWEN) * len(self.ranks_r)
        self.problems = []
        for li in range(layers):
            self.problems.append((RequantProblem * self.nprob)(*[
                RequantProblem(self.W[li][p].data_ptr(), k, self.A[li][r][p].data_ptr(), self.B[li][r][p].data_ptr(),
                               2.0, self.Q[li][r][p].data_ptr(), k, self.S[li][r][p].data_ptr(), n, k, r)
                for p, (_, k, n) in enumerate(QWEN) for r in self.ranks_r]))
        need = max(self.lib.bw_lora_merge_requant_batched_workspace_size(a, self.nprob) for a in self.problems)
        self.ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=dev)  # zero before first use
        self.launches_per_step = 1

    def config(self):
        return workload_config("cfg2", 0)

    variants = QWEN_LAYERS

    def step(self, s, st, events=None):
        li = s % self.layers
        rc = self.lib.bw_lora_merge_requant_batched(self.problems[li], self.nprob, self.ws.data_ptr(),
                                                    self.ws.numel(), st)
        if rc:
            raise RuntimeError(self.lib.bw_last_error().decode())

    # -- end to end through the public API with host (pinned) buffers --
    def e2e_setup(self):
        g = torch.Generator().manual_seed(77 + self.rank)
        self.hW = [(torch.randn((n, k), generator=g) * 0.02).half().pin_memory() for _, k, n in QWEN]
        self.hA = {r: [(torch.randn((r, k), generator=g) / math.sqrt(k)).half().pin_memory() for _, k, n in QWEN]
                   for r in self.ranks_r}
        self.hB = {r: [(torch.randn((n, r), generator=g) * 0.01).half().pin_memory() for _, k, n in QWEN]
                   for r in self.ranks_r}
        self.hQ = {r: [torch.empty((n, k), dtype=torch.int8).pin_memory() for _, k, n in QWEN] for r in self.ranks_r}
        self.hS = {r: [torch.empty((n,), dtype=torch.float16).pin_memory() for _, k, n in QWEN] for r in self.ranks_r}
        self.h2d = sum(t.numel() * 2 for t in self.hW) + sum(
            t.numel() * 2 for r in self.ranks_r for t in self.hA[r] + self.hB[r])
        self.d2h = sum(n * k + 2 * n for _ in self.ranks_r for _, k, n in QWEN)

    def e2e_step(self, s):
        from blackwell_ops.cuda import lora_merge_requant_batched

        W = [t.to(self.dev, non_blocking=True) for t in self.hW]
        A = {r: [t.to(self.dev, non_blocking=True) for t in self.hA[r]] for r in self.ranks_r}
        B = {r: [t.to(self.dev, non_blocking=True) for t in self.hB[r]] for r in self.ranks_r}
        outs = lora_merge_requant_batched([(W[p], A[r][p], B[r][p], 2.0) for p in range(len(QWEN))
                                           for r in self.ranks_r])
        for i, (q, sc) in enumerate(outs):
            p, r = divmod(i, len(self.ranks_r))
            self.hQ[self.ranks_r[r]][p].copy_(q, non_blocking=True)
            self.hS[self.ranks_r[r]][p].copy_(sc, non_blocking=True)

    # -- the reference's CPU PyTorch path on a bounded sample --
    @staticmethod
    def cpu_sample(step_index: int):
        from oracle import torch_port

        _, k, n = QWEN[step_index % len(QWEN)]
        g = torch.Generator().manual_seed(step_index)
        W = (torch.randn((n, k), generator=g) * 0.02).half()
        flops = 0.0
        t0 = time.perf_counter()
        for r in MergeRequantWorkload.ranks_r:
            A = (torch.randn((r, k), generator=g) / math.sqrt(k)).half()
            B = (torch.randn((n, r), generator=g) * 0.01).half()
            t0 = time.perf_counter() if r == MergeRequantWorkload.ranks_r[0] else t0
            torch_port.merge_requant(W, A, B, 2.0)
            flops += 2.0 * r * n * k
        return flops, time.perf_counter() - t0, f"one projection ({n}x{k}) per step, r in {{16,128}}"


class GemmSweepWorkload:
    """cfg1 / cfg3 / cfg3g / cfg4: W8A16 GEMMs through bw_w8a16_gemm (cfg3g: grouped launches through
    bw_w8a16_gemm_grouped) on resident weights."""

    def __init__(self, name, dev, rank, world, m):
        from blackwell_ops import _lib

        self.lib = _lib.lib
        self.dev = dev
        self.name = name
        self.m = m
        self.kernel = "w8a16_persistent_kernel"
        g = torch.Generator(device=dev).manual_seed(2000 + rank)
        if name == "cfg1":
            shapes = [(1024, 3072)] * 64
            self.xdtype = torch.float16
        elif name in ("cfg3", "cfg3g"):
            shapes = [(k, n) for _ in range(QWEN_LAYERS) for _, k, n in QWEN] + [LM_HEAD]
            self.xdtype = torch.float16
        elif name == "cfg4":
            shapes = list(LLAMA8B_MLP)
            self.xdtype = torch.bfloat16
        else:
            raise ValueError(name)
        self.rot = False  # cfg1: one step = 64 GEMMs on 64 distinct weight copies
        self.shapes = shapes
        self.variants = 1
        from blackwell_ops.kernels import quantize_weight_int8

        self.Q, self.S, self.X, self.Y = [], [], [], []
        for k, n in shapes:
            w = randn((n, k), 0.02, self.xdtype, g, dev)
            q, s = quantize_weight_int8(w)
            del w
            self.Q.append(q)
            self.S.append(s)
            self.X.append(randn((m, k), 1.0, self.xdtype, g, dev))
            self.Y.append(torch.empty((m, n), dtype=self.xdtype, device=dev))
        # launches: one GEMM each, or (cfg3g) a layer's q/k/v and gate/up as grouped launches that share
        # their input, as in a decoder layer; o, down and the LM head alone
        if name == "cfg3g":
            self.groups = []
            for li in range(QWEN_LAYERS):
                b = 7 * li
                self.groups += [[b, b + 1, b + 2], [b + 3], [b + 4, b + 5], [b + 6]]
            self.groups.append([len(shapes) - 1])
            for grp in self.groups:
                for i in grp[1:]:
                    self.X[i] = self.X[grp[0]]  # one activation per group
        else:
            self.groups = [[i] for i in range(len(shapes))]
        per = [n * k + 2 * n + 2 * m * n for k, n in shapes]
        per = [v + (2 * m * shapes[i][0] if any(grp[0] == i for grp in self.groups) else 0) for i, v in enumerate(per)]
        fl = [2.0 * m * n * k for k, n in shapes]
        if self.rot:
            self.bytes, self.flops = per[0], fl[0]
            self.launches_per_step = 1
        else:
            self.bytes, self.flops = sum(per), sum(fl)
            self.launches_per_step = len(self.groups)
        self.metric_kind = "tflops" if name == "cfg4" else "gbs"
        self.unit = "TFLOPS" if name == "cfg4" else "GB/s"
        ws = max(self.lib.bw_w8a16_gemm_workspace_size(m, n, k) for k, n in shapes)
        self.cgroups = {}
        for grp in self.groups:
            if len(grp) > 1:
                c = len(grp)
                arr = lambda ct, vals: (ct * c)(*vals)  # noqa: E731
                k = shapes[grp[0]][0]
                ns = arr(ctypes.c_int64, [shapes[i][1] for i in grp])
                self.cgroups[grp[0]] = (c, arr(ctypes.c_void_p, [self.Q[i].data_ptr() for i in grp]),
                                        arr(ctypes.c_int64, [k] * c),
                                        arr(ctypes.c_void_p, [self.S[i].data_ptr() for i in grp]),
                                        arr(ctypes.c_void_p, [self.Y[i].data_ptr() for i in grp]), ns, ns, k)
                ws = max(ws, self.lib.bw_w8a16_gemm_grouped_workspace_size(m, ns, c, k))
        self.ws = torch.zeros(max(ws, 16), dtype=torch.uint8, device=dev)
        self.xcode = 1 if self.xdtype == torch.bfloat16 else 0

    def config(self):
        return workload_config(self.name, self.m)

    def _gemm(self, i, st):
        k, n = self.shapes[i]
        rc = self.lib.bw_w8a16_gemm(self.X[i].data_ptr(), self.xcode, k, self.Q[i].data_ptr(), k, self.S[i].data_ptr(),
                                    self.xcode, self.Y[i].data_ptr(), n, self.m, n, k, self.ws.data_ptr(),
                                    self.ws.numel(), st)
        if rc:
            raise RuntimeError(self.lib.bw_last_error().decode())

    def _grouped(self, i, st):
        c, w, ldw, sc, y, ldy, n, k = self.cgroups[i]
        rc = self.lib.bw_w8a16_gemm_grouped(self.X[i].data_ptr(), self.xcode, k, c, w, ldw, sc, self.xcode, y, ldy, n,
                                            self.m, k, self.ws.data_ptr(), self.ws.numel(), st)
        if rc:
            raise RuntimeError(self.lib.bw_last_error().decode())

    def step(self, s, st, events=None):
        idx = [s % len(self.shapes)] if self.rot else [grp[0] for grp in self.groups]
        for i in idx:
            if events is not None:
                events.append(torch.cuda.Event(enable_timing=True))
                events[-1].record()
            if i in self.cgroups:
                self._grouped(i, st)
            else:
                self._gemm(i, st)
            if events is not None:
                events.append(torch.cuda.Event(enable_timing=True))
                events[-1].record()

    def e2e_setup(self):
        g = torch.Generator().manual_seed(5)
        self.hX = [torch.randn(x.shape, generator=g).to(self.xdtype).pin_memory() for x in self.X]
        self.hY = [torch.empty(y.shape, dtype=self.xdtype).pin_memory() for y in self.Y]
        idx = [0] if self.rot else range(len(self.shapes))
        self.h2d = sum(self.hX[i].numel() * 2 for i in idx if any(grp[0] == i for grp in self.groups))
        self.d2h = sum(self.hY[i].numel() * 2 for i in idx)

    def e2e_step(self, s):
        from blackwell_ops.kernels import int8_gemm, int8_gemm_grouped

        groups = [[s % len(self.shapes)]] if self.rot else self.groups
        for grp in groups:
            x = self.hX[grp[0]].to(self.dev, non_blocking=True)
            if len(grp) == 1:
                ys = [int8_gemm(x, self.Q[grp[0]], self.S[grp[0]])]
            else:
                ys = int8_gemm_grouped(x, [(self.Q[i], self.S[i]) for i in grp])
            for i, y in zip(grp, ys):
                self.hY[i].copy_(y, non_blocking=True)

    def cpu_sample(self, step_index: int):
        from oracle import torch_port

        i = step_index % len(self.shapes)
        k, n = self.shapes[i]
        if self.name in ("cfg4", "cfg5"):
            n = min(n, 1024)  # bounded sample: a 1024-row slice of the projection
        g = torch.Generator().manual_seed(step_index)
        w = (torch.randn((n, k), generator=g) * 0.02).to(self.xdtype)
        q, s = torch_port.quantize_weight_int8(w)
        x = torch.randn((self.m, k), generator=g).to(self.xdtype)
        t0 = time.perf_counter()
        torch_port.int8_gemm(x, q, s)
        dt = time.perf_counter() - t0
        amount = (2.0 * self.m * n * k) if self.metric_kind == "tflops" else (n * k + 2 * n + 2 * self.m * (k + n))
        return amount, dt, f"one projection per step ({n}x{k}, M={self.m})"


class QuantizeWorkload:
    """quant: per-channel int8 quantisation of weights (quantize_weight_int8), HBM-bound.

    One step quantises the Llama-3-8B MLP weights (14336x4096 and 4096x14336, bf16)
    of one of 4 rotating layers (940 MB > L2).  Metric GB/s."""

    kernel = "quantize_rows_stream_kernel"
    name = "quant"
    metric_kind = "gbs"
    unit = "GB/s"

    def __init__(self, dev, rank, world):
        from blackwell_ops import _lib

        self.lib = _lib.lib
        self.dev = dev
        self.xdtype = torch.bfloat16
        g = torch.Generator(device=dev).manual_seed(3000 + rank)
        self.layers = 4
        self.W = [[randn((n, k), 0.02, torch.bfloat16, g, dev) for k, n in LLAMA8B_MLP] for _ in range(self.layers)]
        self.Q = [[torch.empty((n, k), dtype=torch.int8, device=dev) for k, n in LLAMA8B_MLP] for _ in range(self.layers)]
        self.S = [[torch.empty((n,), dtype=torch.bfloat16, device=dev) for k, n in LLAMA8B_MLP] for _ in range(self.layers)]
        self.bytes = sum(2 * n * k + n * k + 2 * n for k, n in LLAMA8B_MLP)
        self.flops = 0.0
        self.variants = self.layers
        self.launches_per_step = len(LLAMA8B_MLP)

    def config(self):
        return workload_config("quant", 0)

    def step(self, s, st, events=None):
        li = s % self.layers
        for j, (k, n) in enumerate(LLAMA8B_MLP):
            rc = self.lib.bw_quantize_rowwise_int8(self.W[li][j].data_ptr(), 1, n, k, k, self.Q[li][j].data_ptr(), k,
                                                   self.S[li][j].data_ptr(), st)
            if rc:
                raise RuntimeError(self.lib.bw_last_error().decode())

    def e2e_setup(self):
        g = torch.Generator().manual_seed(4)
        self.hW = [(torch.randn((n, k), generator=g) * 0.02).bfloat16().pin_memory() for k, n in LLAMA8B_MLP]
        self.hQ = [torch.empty((n, k), dtype=torch.int8).pin_memory() for k, n in LLAMA8B_MLP]
        self.h2d = sum(t.numel() * 2 for t in self.hW)
        self.d2h = sum(n * k + 2 * n for k, n in LLAMA8B_MLP)

    def e2e_step(self, s):
        from blackwell_ops.kernels import quantize_weight_int8

        for j in range(len(LLAMA8B_MLP)):
            q, _ = quantize_weight_int8(self.hW[j].to(self.dev, non_blocking=True))
            self.hQ[j].copy_(q, non_blocking=True)

    @staticmethod
    def cpu_sample(step_index: int):
        from oracle import torch_port

        k, n = LLAMA8B_MLP[step_index % 2]
        n = 1024
        g = torch.Generator().manual_seed(step_index)
        w = (torch.randn((n, k), generator=g) * 0.02).bfloat16()
        t0 = time.perf_counter()
        torch_port.quantize_weight_int8(w)
        return 2 * n * k + n * k + 2 * n, time.perf_counter() - t0, f"1024-row slice of a Llama-3-8B MLP weight (K={k})"


class DeltaWorkload:
    """delta / merge: LoRA delta (lora_delta) or fused merge (lora_merge) at the Llama-3-70B MLP
    shapes (8192->28672, 28672->8192), rank r (default 128), alpha = 2r.  One step computes both
    projections of one of 3 rotating adapters (weights 940 MB > L2).  Metric ΔW TFLOPS; the kernel
    is HBM-bound (it writes N*K fp16), so the roofline is in GB/s."""

    kernel = "lora_stream_kernel"
    metric_kind = "tflops"
    unit = "TFLOPS"

    def __init__(self, name, dev, rank, world, r):
        from blackwell_ops import _lib

        self.lib = _lib.lib
        self.name = name
        self.traffic_key = f"{name}_r{r}"
        self.dev = dev
        self.r = r
        self.xdtype = torch.float16
        g = torch.Generator(device=dev).manual_seed(6000 + rank)
        self.variants = 3
        self.A = [[randn((r, k), 1.0 / math.sqrt(k), torch.float16, g, dev) for k, n in LLAMA70B_MLP]
                  for _ in range(self.variants)]
        self.B = [[randn((n, r), 0.01, torch.float16, g, dev) for k, n in LLAMA70B_MLP] for _ in range(self.variants)]
        self.W = [randn((n, k), 0.02, torch.float16, g, dev) for k, n in LLAMA70B_MLP] if name == "merge" else None
        self.D = [torch.empty((n, k), dtype=torch.float16, device=dev) for k, n in LLAMA70B_MLP]
        self.flops = sum(2.0 * r * n * k for k, n in LLAMA70B_MLP)
        wbytes = 4 if name == "merge" else 2
        self.bytes = sum(wbytes * n * k + 2 * r * (n + k) for k, n in LLAMA70B_MLP)
        self.launches_per_step = len(LLAMA70B_MLP)

    def config(self):
        return {"workload": f"{self.name}: LoRA {'delta' if self.name == 'delta' else 'delta + merge'} at the "
                            f"Llama-3-70B MLP shapes (8192->28672, 28672->8192), r={self.r}, alpha=2r, fp16",
                "r": self.r, "l2": "inputs larger than L2 (3 rotating adapters; the N x K fp16 output is 940 MB)",
                "parallelism": "weak: independent replicas per rank"}

    def step(self, s, st, events=None):
        v = s % self.variants
        for j, (k, n) in enumerate(LLAMA70B_MLP):
            if self.name == "delta":
                rc = self.lib.bw_lora_delta(self.A[v][j].data_ptr(), self.B[v][j].data_ptr(), self.D[j].data_ptr(),
                                            n, k, self.r, 2.0, st)
            else:
                rc = self.lib.bw_lora_merge(self.W[j].data_ptr(), k, self.A[v][j].data_ptr(), self.B[v][j].data_ptr(),
                                            2.0, self.D[j].data_ptr(), k, n, k, self.r, st)
            if rc:
                raise RuntimeError(self.lib.bw_last_error().decode())

    def e2e_setup(self):
        g = torch.Generator().manual_seed(11)
        self.hA = [(torch.randn((self.r, k), generator=g) / math.sqrt(k)).half().pin_memory() for k, n in LLAMA70B_MLP]
        self.hB = [(torch.randn((n, self.r), generator=g) * 0.01).half().pin_memory() for k, n in LLAMA70B_MLP]
        self.hD = [torch.empty((n, k), dtype=torch.float16).pin_memory() for k, n in LLAMA70B_MLP]
        self.h2d = sum(t.numel() * 2 for t in self.hA + self.hB)
        self.d2h = sum(t.numel() * 2 for t in self.hD)

    def e2e_step(self, s):
        from blackwell_ops.cuda import lora_delta, lora_merge

        for j in range(len(LLAMA70B_MLP)):
            A = self.hA[j].to(self.dev, non_blocking=True)
            B = self.hB[j].to(self.dev, non_blocking=True)
            d = lora_delta(A, B, 2.0) if self.name == "delta" else lora_merge(self.W[j], A, B, 2.0)
            self.hD[j].copy_(d, non_blocking=True)

    def cpu_sample(self, step_index: int):
        from oracle import torch_port

        k, n = LLAMA70B_MLP[step_index % 2]
        n = 1024  # bounded sample: a 1024-row slice of the projection
        g = torch.Generator().manual_seed(step_index)
        A = (torch.randn((self.r, k), generator=g) / math.sqrt(k)).half()
        B = (torch.randn((n, self.r), generator=g) * 0.01).half()
        W = (torch.randn((n, k), generator=g) * 0.02).half() if self.name == "merge" else None
        t0 = time.perf_counter()
        d = torch_port.lora_delta(A, B, 2.0)
        if W is not None:
            torch_port.add_delta_(W, d)
        return 2.0 * self.r * n * k, time.perf_counter() - t0, f"1024-row slice of a 70B MLP projection (K={k})"


class NSplitWorkload:
    """cfg5: Llama-3-70B MLP W8A16 with 32 adapter int8 copies, column-parallel over the ranks.

    Setup (adapter load time, not timed): every adapter (r drawn from {16, 64, 128})
    is merged into its own int8 copy of this rank's row shard with
    ``lora_merge_requant_batched``.  A step serves one adapter (round robin):
    the local W8A16 GEMM of each projection writes this rank's slice, NCCL
    all-gathers the slices over NVLink and they are laid out as [M, N].
    """

    kernel = "w8a16_persistent_kernel"
    name = "cfg5"

    def __init__(self, dev, rank, world, m, adapters=32, group=None, gather="fused", xdtype=torch.bfloat16):
        from blackwell_ops import _lib
        from blackwell_ops.cuda import lora_merge_requant_batched
        from blackwell_ops.nsplit import shard_rows

        self.lib = _lib.lib
        self.dev, self.rank, self.world, self.m = dev, rank, world, m
        self.group = group
        self.xdtype = xdtype
        self.shapes = LLAMA70B_MLP  # (K, N)
        g = torch.Generator(device=dev).manual_seed(5000 + rank)
        gr = torch.Generator().manual_seed(77)
        self.ranks_r = [int(v) for v in torch.tensor([16, 64, 128])[torch.randint(0, 3, (adapters,), generator=gr)]]
        self.per = [-(-n // world) for _, n in self.shapes]
        self.Q, self.S = [], []  # [adapter][proj]
        base = []
        for (k, n), per in zip(self.shapes, self.per):
            a, b = shard_rows(n, world, rank)
            w = torch.zeros((per, k), dtype=torch.float16, device=dev)
            w[: b - a] = randn((b - a, k), 0.02, torch.float16, g, dev)
            base.append(w)
        for ai, r in enumerate(self.ranks_r):
            items = []
            for (k, n), per, w in zip(self.shapes, self.per, base):
                A = randn((r, k), 1.0 / math.sqrt(k), torch.float16, g, dev)
                B = randn((per, r), 0.01, torch.float16, g, dev)
                items.append((w, A, B, 2.0))
            outs = lora_merge_requant_batched(items)
            self.Q.append([q for q, _ in outs])
            self.S.append([s for _, s in outs])
        del base
        torch.cuda.synchronize()
        self.X = [randn((m, k), 1.0, self.xdtype, g, dev) for k, _ in self.shapes]
        self.Yloc = [torch.empty((m, per), dtype=self.xdtype, device=dev) for per in self.per]
        self.Ygat = [torch.empty((world, m, per), dtype=self.xdtype, device=dev) for per in self.per]
        self.Y = [torch.empty((m, n), dtype=self.xdtype, device=dev) for _, n in self.shapes]
        ws = max(self.lib.bw_w8a16_gemm_workspace_size(m, per, k) for (k, _), per in zip(self.shapes, self.per))
        self.ws = torch.zeros(max(ws, 16), dtype=torch.uint8, device=dev)
        self.variants = len(self.ranks_r)
        self.launches_per_step = len(self.shapes)
        self.gather = gather if world > 1 else "none"
        self.fused_layers = None
        if self.gather == "fused":
            from blackwell_ops.nsplit import ColumnParallelW8A16

            # one layer per projection; the adapter of a step swaps its weight shard in
            self.fused_layers = [ColumnParallelW8A16(self.Q[0][j], self.S[0][j], n, group=group, fused=True)
                                 for j, (_, n) in enumerate(self.shapes)]
            for j, layer in enumerate(self.fused_layers):
                if not layer.fused:
                    raise SystemExit("cfg5 fused gather needs at least one output column per rank")
                layer.fused_forward(self.X[j], out=self.Y[j])  # sets up the signal pads (collective)
            torch.cuda.synchronize()
        self.metric_kind = "gbs" if m < 512 else "tflops"
        self.unit = "GB/s" if m < 512 else "TFLOPS"
        # whole-job algorithmic work of one step (all ranks together)
        self.bytes_total = sum(n * k + 2 * n + 2 * m * k + 2 * m * n for k, n in self.shapes)
        self.flops_total = sum(2.0 * m * n * k for k, n in self.shapes)
        # this rank's local GEMM work (for the per-kernel roofline)
        self.bytes = sum(per * k + 2 * per + 2 * m * k + 2 * m * per for (k, _), per in zip(self.shapes, self.per))
        self.flops = sum(2.0 * m * per * k for (k, _), per in zip(self.shapes, self.per))

    def config(self):
        c = workload_config("cfg5", self.m) | {"gpus": self.world, "gather": self.gather}
        if self.xdtype == torch.float16:
            c["workload"] = c["workload"].replace("bf16", "f16")
        return c

    def step(self, s, st, events=None):
        ai = s % len(self.ranks_r)
        if self.fused_layers is not None:
            # one kernel per projection, writing the gathered [M, N] output straight into Y
            for j, layer in enumerate(self.fused_layers):
                layer.w, layer.scale = self.Q[ai][j], self.S[ai][j]
                layer.fused_forward(self.X[j], out=self.Y[j])
            return
        for j, ((k, n), per) in enumerate(zip(self.shapes, self.per)):
            # one GPU: straight into Y; N-split with NCCL: into this rank's slice, then gather + relayout
            dst, ld = (self.Y[j], n) if self.world == 1 else (self.Yloc[j], per)
            rc = self.lib.bw_w8a16_gemm(self.X[j].data_ptr(), 1 if self.xdtype == torch.bfloat16 else 0, k,
                                        self.Q[ai][j].data_ptr(), k,
                                        self.S[ai][j].data_ptr(), 0, dst.data_ptr(), ld, self.m, per, k,
                                        self.ws.data_ptr(), self.ws.numel(), st)
            if rc:
                raise RuntimeError(self.lib.bw_last_error().decode())
            if self.world > 1:
                dist.all_gather_into_tensor(self.Ygat[j], self.Yloc[j], group=self.group)
                self.Y[j].copy_(self.Ygat[j].permute(1, 0, 2).reshape(self.m, self.world * per)[:, :n])

    def e2e_setup(self):
        g = torch.Generator().manual_seed(9)
        self.hX = [torch.randn(x.shape, generator=g).to(self.xdtype).pin_memory() for x in self.X]
        self.hY = [torch.empty(y.shape, dtype=self.xdtype).pin_memory() for y in self.Y]
        self.h2d = sum(x.numel() * 2 for x in self.hX)
        self.d2h = sum(y.numel() * 2 for y in self.hY)

    def e2e_step(self, s):
        from blackwell_ops.nsplit import ColumnParallelW8A16

        ai = s % len(self.ranks_r)
        for j, (k, n) in enumerate(self.shapes):
            x = self.hX[j].to(self.dev, non_blocking=True)
            if self.fused_layers is not None:
                layer = self.fused_layers[j]
                layer.w, layer.scale = self.Q[ai][j], self.S[ai][j]
            else:
                layer = ColumnParallelW8A16(self.Q[ai][j], self.S[ai][j], n, group=self.group)
            self.hY[j].copy_(layer(x), non_blocking=True)

    def cpu_sample(self, step_index: int):
        from oracle import torch_port

        k, n = self.shapes[step_index % 2]
        n = 1024  # bounded sample: a 1024-row slice of the projection
        g = torch.Generator().manual_seed(step_index)
        w = (torch.randn((n, k), generator=g) * 0.02).half()
        q, s = torch_port.quantize_weight_int8(w)
        x = torch.randn((self.m, k), generator=g).to(self.xdtype)
        t0 = time.perf_counter()
        torch_port.int8_gemm(x, q, s)
        dt = time.perf_counter() - t0
        amount = (2.0 * self.m * n * k) if self.metric_kind == "tflops" else (n * k + 2 * n + 2 * self.m * (k + n))
        return amount, dt, f"1024-row slice of a 70B MLP projection per step (K={k}, M={self.m})"


# ---------------------------------------------------------------------------
# main
# ---------------------------------------------------------------------------
def make_workload(args, dev, rank, world):
    if args.workload == "cfg2":
        return MergeRequantWorkload(dev, rank, world)
    if args.workload in ("cfg1", "cfg3", "cfg3g", "cfg4"):
        m = args.m if args.m else {"cfg1": 16, "cfg3": 16, "cfg3g": 16, "cfg4": 2048}[args.workload]
        return GemmSweepWorkload(args.workload, dev, rank, world, m)
    if args.workload == "quant":
        return QuantizeWorkload(dev, rank, world)
    if args.workload in ("delta", "merge"):
        return DeltaWorkload(args.workload, dev, rank, world, args.rank)
    if args.workload == "cfg5":
        return NSplitWorkload(dev, rank, world, args.m if args.m else 16, adapters=args.adapters,
                              gather=args.gather, xdtype=torch.float16 if args.dtype == "f16" else torch.bfloat16)
    raise SystemExit(f"unknown workload {args.workload}")


def summarize_phases(launches, per_step: int) -> dict:
    """Median over the traced steps of each GEMM launch's phase ends (us from its first CTA
    start) and of the gap from one launch's last phase to the next launch's first CTA start."""
    import statistics

    rows = [l.phases_us() for l in launches]
    ends = []
    for l in launches:
        st = l.stamps.double()
        ends.append((float(st[:, 0][st[:, 0] > 0].min()), float(st.max())))
    out = {"launches_traced": len(rows), "per_launch_us": {}}
    keys = sorted({k for r in rows for k in r})
    for k in keys:
        vals = [r[k] for r in rows if k in r]
        out["per_launch_us"][k] = round(statistics.median(vals), 3)
    gaps = [(ends[i + 1][0] - ends[i][1]) / 1e3 for i in range(len(ends) - 1)]
    if gaps:
        out["gap_between_launches_us"] = round(statistics.median(gaps), 3)
    durs = [(e - b) / 1e3 for b, e in ends]
    out["launch_span_us"] = round(statistics.median(durs), 3)
    return out


def amount_of(wl) -> float:
    return wl.flops if wl.metric_kind == "tflops" else wl.bytes


def scale_unit(amount: float, seconds: float, kind: str) -> float:
    return amount / seconds / (1e12 if kind == "tflops" else 1e9)


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU PyTorch path (oracle port) on the host cores."""
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    cores = torch.get_num_threads()
    if args.workload == "cfg2":
        sample = MergeRequantWorkload.cpu_sample
        kind, unit = "tflops", "TFLOPS"
    elif args.workload == "quant":
        sample = QuantizeWorkload.cpu_sample
        kind, unit = "gbs", "GB/s"
    elif args.workload in ("delta", "merge"):
        sample = lambda i: DeltaWorkload.cpu_sample(argparse.Namespace(r=args.rank, name=args.workload), i)
        kind, unit = "tflops", "TFLOPS"
    else:
        wl_cpu = GemmCpuShim(args)
        sample, kind, unit = wl_cpu.cpu_sample, wl_cpu.metric_kind, wl_cpu.unit
    for i in range(args.warmup):
        sample(i)
    tot, secs, desc = 0.0, 0.0, ""
    for i in range(args.steps):
        a, t, desc = sample(args.warmup + i)
        tot += a
        secs += t
    v = scale_unit(tot, secs, kind)
    line = {"impl": "reference", "metric": METRIC, "value": round(v, 6), "unit": unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(secs / args.steps * 1e3, 3),
            "higher_is_better": True, "scaling": "strong" if args.workload == "cfg5" else "weak", "vs_baseline": None,
            "dtype": "bf16" if args.workload in ("cfg4", "cfg5") else "f16",
            "data": "synthetic (seeded), random-init weights",
            "config": config_for(args),
            "cpu_baseline": {"value": round(v, 6), "unit": unit, "cores": cores, "kind": "port", "sample": desc},
            "e2e": {"value": round(v, 6), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


class GemmCpuShim:
    """CPU-only view of a GEMM workload's shapes for the reference arm (no GPU state)."""

    def __init__(self, args):
        self.name = args.workload
        self.m = args.m if args.m else DEFAULT_M.get(args.workload, 16)
        self.xdtype = torch.bfloat16 if self.name == "cfg4" else torch.float16
        if self.name == "cfg1":
            self.shapes = [(1024, 3072)]
        elif self.name in ("cfg3", "cfg3g"):
            self.shapes = [(k, n) for _, k, n in QWEN] + [LM_HEAD]
        elif self.name == "cfg5":
            self.shapes = list(LLAMA70B_MLP)
            self.xdtype = torch.bfloat16
        else:
            self.shapes = list(LLAMA8B_MLP)
        big_m = self.name == "cfg4" or (self.name == "cfg5" and self.m >= 512)
        self.metric_kind = "tflops" if big_m else "gbs"
        self.unit = "TFLOPS" if big_m else "GB/s"

    cpu_sample = GemmSweepWorkload.cpu_sample


METRIC = "W8A16 GEMM HBM GB/s (decode) / TFLOPS (prefill, ΔW) vs B200 roofline"

DEFAULT_M = {"cfg1": 16, "cfg3": 16, "cfg3g": 16, "cfg4": 2048, "cfg5": 16}


def workload_config(name: str, m: int) -> dict:
    """The `config` object of the JSON line; identical for both arms."""
    if name == "quant":
        return {"workload": "quant: quantize_weight_int8 of Llama-3-8B MLP weights (14336x4096, 4096x14336), bf16",
                "l2": "inputs larger than L2 (4 rotating layers, 940 MB)", "parallelism": "weak: independent replicas"}
    if name == "cfg2":
        return {"workload": "cfg2: LoRA delta+merge+requant, Qwen3-0.6B layer (7 projections), r in {16,128}, "
                            "alpha=2r (scaling 2)", "layers_rotated": QWEN_LAYERS,
                "l2": "inputs larger than L2: each step merges a different layer (28 layers, 412 MB fp16 W)",
                "parallelism": "weak: each rank merges its own layers, no collective"}
    m = m or DEFAULT_M[name]
    desc = {"cfg1": "cfg1: W8A16 GEMM X[16,1024] x W[3072,1024]^T, fp16; one step = 64 GEMMs on 64 distinct "
                    "weight copies (210 MB > L2)",
            "cfg3": f"cfg3: Qwen3-0.6B decode sweep, 28 layers x 7 projections + LM head, M={m}, fp16",
            "cfg3g": f"cfg3g: the cfg3 sweep with each layer's q/k/v and gate/up as grouped launches sharing their "
                     f"input (4 launches per layer), M={m}, fp16",
            "cfg4": f"cfg4: Llama-3-8B MLP prefill W8A16 (4096->14336, 14336->4096), M={m}, bf16",
            "cfg5": f"cfg5: Llama-3-70B MLP W8A16 (8192->28672, 28672->8192), 32 adapter int8 copies "
                    f"(r in {{16,64,128}}), M={m}, bf16"}[name]
    if name == "cfg5":
        return {"workload": desc, "m": m, "l2": "inputs larger than L2: a step streams 470 MB of int8 weights (470/N MB per rank) of one of "
                "32 adapter copies in turn, so a weight byte is re-read only after 31 other adapters' steps "
                "(>= 1.8 GB per rank at N = 8)",
                "parallelism": "column-parallel N-split over the GPUs, output slices all-gathered inside the GEMM "
                               "epilogue over peer memory (--gather fused) or by NCCL (--gather nccl); strong"}
    return {"workload": desc, "m": m, "l2": "inputs larger than L2 (weights streamed from HBM each step)",
            "parallelism": "weak: independent replicas per rank"}


def config_for(args, wl=None):
    if wl is not None:
        return wl.config()
    if args.workload in ("delta", "merge"):
        return DeltaWorkload.config(argparse.Namespace(r=args.rank, name=args.workload))
    return workload_config(args.workload, args.m)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", default="cfg5")
    ap.add_argument("--trace", action="store_true", help="add device-side phase stamps of a few steps")
    ap.add_argument("--m", type=int, default=0, help="tokens for the GEMM workloads")
    ap.add_argument("--adapters", type=int, default=32, help="cfg5: number of adapters")
    ap.add_argument("--rank", type=int, default=128, help="delta / merge: LoRA rank r")
    ap.add_argument("--gather", choices=("fused", "nccl"), default="fused",
                    help="cfg5 on several GPUs: all-gather inside the GEMM epilogue over peer memory, or NCCL")
    ap.add_argument("--dtype", choices=("bf16", "f16"), default="bf16", help="cfg5: activation dtype")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    wl = make_workload(args, dev, rank, world)
    st_ptr = torch.cuda.current_stream(dev).cuda_stream
    peaks = load_peaks()

    # ---- eager pass over every distinct step (kernel attributes, status), then CUDA graphs of
    # consecutive steps: a graph holds a run of steps back to back, as a serving runtime captures a
    # whole decode step, so each kernel's programmatic dependent launch overlaps its start with the
    # end of the kernel before it, across step boundaries too ----
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for v in range(wl.variants):
            wl.step(v, side.cuda_stream)
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize()
    offset = 7 * rank
    graphs = []

    def capture(first: int, count: int):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for s in range(first, first + count):
                wl.step((s + offset) % wl.variants, torch.cuda.current_stream(dev).cuda_stream)
        graphs.append(g)
        return g

    warm = capture(0, args.warmup)
    timed = capture(args.warmup, args.steps)  # exactly the K timed steps
    upload_graph(timed, torch.cuda.current_stream(dev))  # its first launch would otherwise upload it
    warm.replay()
    torch.cuda.synchronize()
    barrier()

    # ---- timed region: one replay of the K-step graph ----
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(gpu_index(local))
    barrier()
    torch.cuda.synchronize()
    with sampler:
        start.record()
        timed.replay()
        end.record()
        torch.cuda.synchronize()
    barrier()
    ms = start.elapsed_time(end)
    ms_max = max_over_ranks(ms)

    # ---- dominant-kernel duration: every kernel of a step is the dominant kernel, so CUDA events
    # (on the launching stream) around a second replay of the K steps give the launches' duration,
    # overlap with their neighbours included ----
    a_ev, b_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a_ev.record()
    timed.replay()
    b_ev.record()
    torch.cuda.synchronize()
    kern_ms = a_ev.elapsed_time(b_ev)
    n_launch = wl.launches_per_step * args.steps
    kern_ms_per_step = kern_ms / args.steps

    amount = amount_of(wl)
    if wl.name == "cfg5":  # strong scaling: the job's work is fixed, shared by the ranks
        amount = wl.flops_total if wl.metric_kind == "tflops" else wl.bytes_total
        value = scale_unit(amount, ms_max / args.steps / 1e3, wl.metric_kind)
    else:
        value = scale_unit(amount * world, ms_max / args.steps / 1e3, wl.metric_kind)
    achieved_gbs = wl.bytes / (kern_ms_per_step / 1e3) / 1e9
    achieved_tf = wl.flops / (kern_ms_per_step / 1e3) / 1e12
    if wl.name == "cfg4" or (wl.name in ("cfg5",) and wl.metric_kind == "tflops"):
        roof = {"bound": "tensor", "achieved": round(achieved_tf, 2), "peak": peaks["bf16_tflops"],
                "unit": "TFLOP/s", "frac": round(achieved_tf / peaks["bf16_tflops"], 4)}
    else:
        roof = {"bound": "hbm", "achieved": round(achieved_gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": round(achieved_gbs / peaks["hbm_gbs"], 4)}
    roof["peak_source"] = peaks["source"] + " (MEASURED_PEAKS.json)" if peaks["source"] == "measured" else "fallback"
    # the same fraction against the spec peaks north_star names (HBM ~8 TB/s, dense bf16 2.25 PFLOP/s)
    roof["spec_peak"] = 8000.0 if roof["unit"] == "GB/s" else 2250.0
    roof["frac_of_spec"] = round(roof["achieved"] / roof["spec_peak"], 4)
    roof["traffic"] = load_traffic(wl.kernel, getattr(wl, "traffic_key", wl.name))
    roof["kernel"] = wl.kernel
    roof["launches_timed"] = n_launch
    roof["timing"] = ("CUDA events around one replay of a CUDA graph of the K steps (kernels chained by "
                      "programmatic dependent launch); includes inter-kernel gaps")
    roof["bytes_per_step"] = wl.bytes
    if wl.metric_kind == "tflops" and roof["bound"] == "hbm":
        roof["tensor_tflops"] = round(achieved_tf, 2)

    # ---- device-side phase stamps of a few replayed steps (--trace) ----
    phases = None
    if args.trace:
        from blackwell_ops.device import Trace

        tg = capture(0, 4)
        with Trace(records=4096, device=dev) as tr:
            tg.replay()
        phases = summarize_phases(tr.launches(), wl.launches_per_step)

    # ---- end to end through the public API, host buffers ----
    e2e = None
    if not args.no_e2e:
        wl.e2e_setup()
        for s in range(args.warmup):
            wl.e2e_step(s)
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for s in range(args.steps):
            wl.e2e_step(s)
        e1.record()
        torch.cuda.synchronize()
        barrier()
        e_ms = max_over_ranks(e0.elapsed_time(e1))
        e2e_amount = amount if wl.name == "cfg5" else amount * world
        e2e = {"value": round(scale_unit(e2e_amount, e_ms / args.steps / 1e3, wl.metric_kind), 4),
               "unit": wl.unit, "h2d_bytes_per_step": wl.h2d, "d2h_bytes_per_step": wl.d2h,
               "ms_per_step": round(e_ms / args.steps, 4)}

    from blackwell_ops import _lib

    status = _lib.device_status(clear=False)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        torch.set_num_threads(os.cpu_count() or 1)
        tot, secs, i, desc = 0.0, 0.0, 0, ""
        while secs < 10.0 and i < 64:
            a, t, desc = wl.cpu_sample(i)
            if i > 0:  # first call warms the CPU path
                tot += a
                secs += t
            i += 1
        cpu = {"value": round(scale_unit(tot, secs, wl.metric_kind), 6), "unit": wl.unit,
               "cores": torch.get_num_threads(), "kind": "port", "sample": desc + f", {i - 1} samples"}

    for g in graphs:  # graphs holding NCCL work are released before the process group
        g.reset()
    graphs.clear()
    torch.cuda.synchronize()
    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 4), "unit": wl.unit, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True,
                "scaling": "strong" if wl.name == "cfg5" else "weak", "vs_baseline": None,
                "dtype": "bf16" if getattr(wl, "xdtype", torch.float16) == torch.bfloat16 else "f16",
                "data": "synthetic (seeded), random-init weights", "config": wl.config(), "roofline": roof,
                "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": wl.launches_per_step * args.steps,
                "clocks": sampler.summary(), "device_status": status}
        if phases is not None:
            line["phases"] = phases
        print(json.dumps(line), flush=True)
    if world > 1:
        # Teardown order: every CUDA graph (some hold NCCL work) was reset above; the workload's
        # layers hold symmetric-memory signal pads, which are released here, on every rank, before
        # the last collective and destroy_process_group (a symmetric-memory handle still alive at
        # destroy is the remaining suspect of the one teardown that hung)
        import gc

        del wl
        gc.collect()
        torch.cuda.synchronize()
        # the result is out; bound the teardown so a stuck communicator cannot hold the GPUs
        import threading

        def _bail_timeout():
            # the JSON line is out, but a teardown that does not finish is a failure of the run
            sys.stdout.flush()
            sys.stderr.write(f"rank {rank}: teardown timeout (barrier / destroy_process_group did not finish "
                             f"within 60 s)\n")
            sys.stderr.flush()
            os._exit(3)

        guard = threading.Timer(60.0, _bail_timeout)
        guard.daemon = True
        guard.start()
        barrier()
        dist.destroy_process_group()
        guard.cancel()


if __name__ == "__main__":
    main()
