"""Column-parallel (N-split) W8A16 linear over one node's GPUs.

The reference has no multi-GPU code.  This is the north star's partitioning
of large projections: rank g of G owns output rows [g*Ns, (g+1)*Ns) of the
int8 weight and its per-channel scale (Ns = ceil(N / G)); activations are
replicated.  Each rank runs the local W8A16 GEMM into its slice of the
all-gather buffer, NCCL all-gathers the G slices over NVLink into
[G, M, Ns], and the slices are laid out as [M, N].

Per-channel quantisation and the LoRA merge / requantisation are shard-local
(a row's scale depends only on that row), so adapters are merged into each
rank's shard with no communication: ``shard_rows`` gives the row range, and
``blackwell_ops.cuda.lora_merge_requant(W[rows], A, B[rows], s)`` produces
the rank's int8 copy.

The local GEMM is a parameter so the sharding / gather logic can be exercised
on CPU ranks (gloo) with any function of the same signature; the default is
the tcgen05 kernel.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist


def shard_rows(n: int, world: int, rank: int) -> tuple[int, int]:
    """Row range [start, stop) of rank `rank`; every shard is padded to ceil(n/world) rows."""
    per = -(-n // world)
    start = min(rank * per, n)
    return start, min(start + per, n)


def shard_weight(w_int8: torch.Tensor, scale: torch.Tensor, world: int, rank: int):
    """This rank's rows of (w_int8 [N, K], scale [N]), zero-padded to ceil(N/world) rows."""
    n = w_int8.shape[0]
    per = -(-n // world)
    start, stop = shard_rows(n, world, rank)
    q = torch.zeros((per, w_int8.shape[1]), dtype=w_int8.dtype, device=w_int8.device)
    s = torch.zeros((per,), dtype=scale.dtype, device=scale.device)
    if stop > start:
        q[: stop - start].copy_(w_int8[start:stop])
        s[: stop - start].copy_(scale[start:stop])
    return q, s


def _default_gemm():
    from .kernels import int8_gemm

    return int8_gemm


class ColumnParallelW8A16:
    """y = x @ (w_int8 * scale).T with w's rows split across the ranks of `group`."""

    def __init__(self, w_shard: torch.Tensor, scale_shard: torch.Tensor, n_total: int,
                 group: dist.ProcessGroup | None = None,
                 local_gemm: Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor] | None = None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        per = -(-n_total // self.world)
        if w_shard.shape[0] != per or scale_shard.shape[0] != per:
            raise RuntimeError(f"shard must hold ceil(N/G) = {per} rows (got {w_shard.shape[0]})")
        self.w = w_shard
        self.scale = scale_shard
        self.n_total = n_total
        self.per = per
        self.local_gemm = local_gemm or _default_gemm()
        self._use_into_tensor = True

    def local(self, x: torch.Tensor) -> torch.Tensor:
        return self.local_gemm(x, self.w, self.scale)

    def gather(self, y_local: torch.Tensor) -> torch.Tensor:
        """[M, Ns] per rank -> [M, N] on every rank."""
        m = y_local.shape[0]
        if self.world == 1:
            return y_local[:, : self.n_total]
        buf = torch.empty((self.world, m, self.per), dtype=y_local.dtype, device=y_local.device)
        y_local = y_local.contiguous()
        if self._use_into_tensor:
            try:
                dist.all_gather_into_tensor(buf, y_local, group=self.group)
            except (RuntimeError, NotImplementedError, AttributeError):
                self._use_into_tensor = False
        if not self._use_into_tensor:
            dist.all_gather(list(buf.unbind(0)), y_local, group=self.group)
        return buf.permute(1, 0, 2).reshape(m, self.world * self.per)[:, : self.n_total]

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return self.gather(self.local(x))
