"""Column-parallel N-split on CPU ranks (gloo, world size 2 and 3).

The sharding, the per-shard requantisation independence and the all-gather +
relayout run exactly as on GPUs; only the local GEMM is the oracle's CPU
dequantise-matmul (the product path uses the tcgen05 kernel).  Also covers a
rank that fails before the collective: the others see an error, not a hang.
"""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cpu_gemm(x, q, s):
    from oracle import torch_port

    return torch_port.int8_gemm(x, q, s)


def _worker(rank, world, port, n, k, m, out_dir, fail_rank):
    sys.path[:0] = [str(ROOT), str(ROOT / "blackwell-inference-server_b200")]
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        from blackwell_ops.nsplit import ColumnParallelW8A16, shard_rows, shard_weight
        from oracle import torch_port

        g = torch.Generator().manual_seed(123)
        w = (torch.randn(n, k, generator=g) * 0.02).half()
        x = torch.randn(m, k, generator=g).half()
        q_full, s_full = torch_port.quantize_weight_int8(w)
        # shard-local quantisation equals slicing the full quantisation (per-channel)
        a, b = shard_rows(n, world, rank)
        q_loc, s_loc = torch_port.quantize_weight_int8(w[a:b])
        assert torch.equal(q_loc, q_full[a:b]) and torch.equal(s_loc, s_full[a:b])
        qs, ss = shard_weight(q_full, s_full, world, rank)
        layer = ColumnParallelW8A16(qs, ss, n, local_gemm=_cpu_gemm)
        if rank == fail_rank:
            raise SystemExit(3)  # leaves before the collective
        y = layer(x)
        ref = torch_port.int8_gemm(x, q_full, s_full)
        torch.save({"y": y, "ref": ref}, Path(out_dir) / f"r{rank}.pt")
    except Exception as e:  # reported to the parent through the exit code
        (Path(out_dir) / f"err{rank}.txt").write_text(repr(e))
        raise
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("world,n", [(2, 3072), (3, 1000)])
def test_nsplit_gather_matches_unsplit(world, n, tmp_path):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n, 256, 5, str(tmp_path), -1)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0, (p.exitcode, [f.read_text() for f in tmp_path.glob("err*.txt")])
    for r in range(world):
        d = torch.load(tmp_path / f"r{r}.pt")
        assert d["y"].shape == (5, n)
        assert torch.equal(d["y"], d["ref"])


def test_nsplit_rank_failure_is_an_error_not_a_hang(tmp_path):
    ctx = mp.get_context("spawn")
    port = _free_port()
    world = 2
    procs = [ctx.Process(target=_worker, args=(r, world, port, 512, 64, 2, str(tmp_path), 1)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
        assert p.exitcode is not None, "a rank hung"
    assert procs[1].exitcode == 3
    assert procs[0].exitcode != 0  # the survivor's collective failed instead of waiting forever


def test_shard_rows_cover_every_row():
    from blackwell_ops.nsplit import shard_rows

    for n in (1, 7, 8192, 28672, 151936):
        for world in (1, 2, 3, 4, 8):
            covered = []
            for r in range(world):
                a, b = shard_rows(n, world, r)
                covered.extend(range(a, b))
            assert covered == list(range(n))
