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

``fused=True`` replaces GEMM + NCCL all-gather by one kernel per rank
(``bw_w8a16_gemm_allgather``) for M <= 256: each rank's epilogue stores its
output tiles into its own [M, N] output and sends them to every peer's
signal-pad mailbox (a symmetric-memory buffer, plain stores over NVLink of
8-byte words that carry the call's epoch, so no fence or flag handshake is
needed); each rank copies its peers' tiles into its output as they arrive.  It
needs CUDA ranks on one node and at least one output column per rank;
otherwise, and for M > 256, the NCCL path runs.  ``check=True`` synchronises
after each call and raises ``DeviceTimeoutError`` if a wait for a peer ran out
(a rank that did not make the same call); the layer's signal pads must then be
reset with ``reset()`` on every rank before its next call.
"""
from __future__ import annotations

import ctypes
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
                 local_gemm: Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor] | None = None,
                 fused: bool = False, check: bool = False):
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
        # fused all-gather: CUDA ranks with the library's kernel (the same decision on all ranks)
        self.fused = fused and self.world > 1 and local_gemm is None and w_shard.is_cuda
        self._symm: dict = {}
        self.check = check

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

    def _signal_pads(self, m: int, device: torch.device):
        """Symmetric signal pads for calls with this M (a collective on first use)."""
        st = self._symm.get(m)
        if st is None:
            import torch.distributed._symmetric_memory as symm_mem

            from ._lib import lib

            group = self.group if self.group is not None else dist.group.WORLD
            enable = getattr(symm_mem, "enable_symm_mem_for_group", None)
            if enable is not None:
                enable(group.group_name)
            nbytes = lib.bw_w8a16_gemm_allgather_signal_bytes(m, self.per, self.world)
            sig = symm_mem.empty(((nbytes + 15) // 16 * 4,), dtype=torch.int32, device=device)
            sig.zero_()
            hs = symm_mem.rendezvous(sig, group.group_name)
            torch.cuda.synchronize(device)
            dist.barrier(group=group)  # every rank's pad is zero before anyone sends
            sp = (ctypes.c_void_p * self.world)(*[int(p) for p in hs.buffer_ptrs])
            st = self._symm[m] = (sig, hs, sp, sig.numel() * 4)
        return st

    def fused_forward(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """One kernel per rank: local GEMM with the all-gather over peer memory in its epilogue."""
        from ._lib import DTYPE_CODE, GATHER_MAX_M, check, lib, stream_ptr
        from .kernels.int8_gemm import _workspace

        if x.dim() != 2 or x.dtype not in (torch.float16, torch.bfloat16):
            raise RuntimeError("fused N-split: x must be a 2-D fp16 or bf16 tensor")
        if x.stride(1) != 1:
            x = x.contiguous()
        m, k = x.shape
        if m > GATHER_MAX_M or m == 0:
            y = self.gather(self.local(x))
            if out is not None:
                out.copy_(y)
                return out
            return y
        # every rank computes its whole padded shard (per rows; the rows past N are zero weights
        # whose outputs land in the padding columns), so all ranks run the same plan
        _, _, sp, nbytes = self._signal_pads(m, x.device)
        ld = self.world * self.per
        if out is not None and out.shape == (m, self.n_total) and out.dtype == x.dtype and out.stride() == (ld, 1):
            y, ret = out, out
        else:
            y = torch.empty((m, ld), dtype=x.dtype, device=x.device)
            ret = None
        st = stream_ptr(x.device)
        need = lib.bw_w8a16_gemm_allgather_workspace_size(m, self.per, k)
        ws = _workspace(x.device, st, need)
        with torch.cuda.device(x.device):
            check(lib.bw_w8a16_gemm_allgather(
                x.data_ptr(), DTYPE_CODE[x.dtype], x.stride(0), self.w.data_ptr(), self.w.stride(0),
                self.scale.data_ptr(), DTYPE_CODE[self.scale.dtype], y.data_ptr(), ld, self.rank * self.per,
                m, self.per, k, sp, nbytes, self.world, self.rank, ws.data_ptr() if ws is not None else None,
                ws.numel() if ws is not None else 0, st), "int8_gemm (all-gather)")
        if self.check:
            from .device import check

            check(x.device, "int8_gemm (all-gather)")
        if ret is not None:
            return ret
        if out is not None:
            out.copy_(y[:, : self.n_total])
            return out
        return y[:, : self.n_total]

    def reset(self) -> None:
        """Zero this rank's signal pads (collective: every rank calls it, e.g. after a timeout)."""
        if not self._symm:
            return
        group = self.group if self.group is not None else dist.group.WORLD
        for (sig, _, _, _) in self._symm.values():
            sig.zero_()
        torch.cuda.synchronize()
        dist.barrier(group=group)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if self.fused:
            return self.fused_forward(x)
        return self.gather(self.local(x))
