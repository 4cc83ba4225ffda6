"""Column-parallel N-split on real GPUs: one process per GPU, NCCL all-gather.

Each rank quantises its row shard of the weight on its own GPU, runs the
tcgen05 W8A16 GEMM on it, and the slices are all-gathered over NVLink into
[M, N], once with NCCL and once by the fused kernel that sends its tiles to
every peer's signal-pad mailbox over peer memory (M <= 256; larger M takes
the NCCL path inside the same layer).  The result must equal the single-GPU GEMM of the full weight within
the GEMM tolerance (max |err| <= 1e-2, relative <= 1e-3 against the fp32
dequantise-matmul) and, row for row, the codes and scales of the full
quantisation.  Runs at world sizes 2, 4 and 8, each where that many GPUs are
visible (skipped otherwise).
"""
import os
import socket
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

ROOT = Path(__file__).resolve().parent.parent


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, cases, out_dir):
    sys.path[:0] = [str(ROOT), str(ROOT / "blackwell-inference-server_b200")]
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import datetime

    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    failures = []
    from blackwell_ops import _lib
    from blackwell_ops.kernels import int8_gemm, quantize_weight_int8
    from blackwell_ops.nsplit import ColumnParallelW8A16, shard_rows

    for m, n, k, dt in cases:
        # every rank takes the same collective steps even when a check fails: the
        # ranks agree that their shards are ready before the all-gather
        dtype = torch.float16 if dt == "f16" else torch.bfloat16
        layer = x = w = None
        ready = torch.ones(1, device=dev)
        try:
            g = torch.Generator(device=dev).manual_seed(1000 + m + n + k)
            w = (torch.randn(n, k, generator=g, device=dev) * 0.02).to(dtype)  # every rank draws the full weight
            x = torch.randn(m, k, generator=g, device=dev).to(dtype)
            a, b = shard_rows(n, world, rank)
            per = -(-n // world)
            q_loc = torch.zeros((per, k), dtype=torch.int8, device=dev)
            s_loc = torch.zeros((per,), dtype=dtype, device=dev)
            if b > a:
                q, s = quantize_weight_int8(w[a:b].contiguous())  # shard-local quantisation
                q_loc[: b - a].copy_(q)
                s_loc[: b - a].copy_(s)
            layer = ColumnParallelW8A16(q_loc, s_loc, n)
            y_loc = layer.local(x)
            torch.cuda.synchronize()
        except Exception as e:
            failures.append(f"case {(m, n, k, dt)} prepare: {type(e).__name__}: {e}")
            ready.zero_()
        dist.all_reduce(ready, op=dist.ReduceOp.MIN)
        if float(ready) == 0.0:
            continue
        y = layer.gather(y_loc)
        torch.cuda.synchronize()
        # the fused kernel (all-gather over peer memory in the GEMM epilogue): same result on every
        # rank, on two calls in a row and from a replayed CUDA graph (the epoch lives on the device)
        fused = ColumnParallelW8A16(q_loc, s_loc, n, fused=True)
        outs = [fused(x), fused(x)]
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            yg = fused(x)
        for _ in range(2):
            gr.replay()
        torch.cuda.synchronize()
        outs.append(yg.clone())
        # drop the graph (and its output) here, outside any capture
        del gr, yg
        try:
            assert fused.fused, "fused path not taken"
            for i, yf in enumerate(outs):
                bound = 1e-2 + 2.0 ** (-10 if dt == "f16" else -7) * y.float().abs()
                d = (yf.float() - y.float()).abs()
                assert bool((d <= bound).all()), f"fused call {i}: |fused - nccl| up to {float(d.max())}"
        except Exception as e:
            failures.append(f"case {(m, n, k, dt)} fused: {type(e).__name__}: {e}")
        del outs, fused
        torch.cuda.synchronize()
        if rank == 0:
            try:
                q_full, s_full = quantize_weight_int8(w)
                assert torch.equal(q_loc[: b - a], q_full[a:b]) and torch.equal(s_loc[: b - a], s_full[a:b]), \
                    "shard-local codes differ from the full quantisation"
                ref32 = x.float() @ (q_full.float() * s_full.float()[:, None]).t()
                assert y.shape == (m, n), f"shape {tuple(y.shape)}"
                tol = 1e-2 if dt == "f16" else 1e-2 + 2 ** -8 * float(ref32.abs().max())
                e = float((y.float() - ref32).abs().max())
                assert e <= tol, f"max |err| {e} > {tol}"
                rel = float((y.float() - ref32).norm() / ref32.norm())
                assert rel <= (1e-3 if dt == "f16" else 4e-3), f"relative err {rel}"
                # the unsplit GEMM may sum in another split-K order: within the GEMM bar plus one output ulp
                y1 = int8_gemm(x, q_full, s_full)
                bound = 1e-2 + 2.0 ** (-10 if dt == "f16" else -7) * y1.float().abs()
                d = (y.float() - y1.float()).abs()
                assert bool((d <= bound).all()), f"|split - unsplit| up to {float(d.max())}"
            except Exception as e:
                failures.append(f"case {(m, n, k, dt)} check: {type(e).__name__}: {e}")
    if _lib.device_status() != 0:
        failures.append(f"device status {_lib.device_status()}")
    status = "ok" if not failures else f"rank {rank}: " + "; ".join(failures)
    Path(out_dir, f"rank{rank}.txt").write_text(status)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_column_parallel_nccl_matches_single_gpu(tmp_path, world):
    import torch.multiprocessing as mp

    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    cases = [(16, 3072, 1024, "f16"), (1, 1000, 512, "f16"), (64, 28672 // 8, 8192, "bf16"), (300, 4096, 1024, "bf16"),
             (16, 1003, 2048, "bf16"), (256, 2048, 1024, "f16"), (7, 28672, 8192, "bf16")]
    mp.spawn(_worker, args=(world, _free_port(), cases, str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        assert Path(tmp_path, f"rank{r}.txt").read_text() == "ok"
